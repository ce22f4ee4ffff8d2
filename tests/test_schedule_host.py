"""Host logic on the CPU: the pipelined pass A / pass B order of a streamed pair list (engine.pipeline_steps), the
symmetric-contraction coefficient layout the kernels read four at a time (engine.sc_coef_layout), and LAMMPS's
spatial atom sort (structures.lammps_bin_order)."""
import numpy as np
import pytest

from mace_onegpu import engine as E
from mace_onegpu import structures as S


def _run(nch, chunk, nl, his, lookahead=2):
    """The yielded steps, and for every largest_sender call the number of pass-A chunks issued before it."""
    steps, calls = [], []
    n_a = [0]

    def largest_sender(c):
        calls.append((c, n_a[0]))
        return his[c]

    for kind, k in E.pipeline_steps(nch, chunk, nl, largest_sender, lookahead):
        steps.append((kind, k))
        n_a[0] += kind == "A"
    return steps, calls


def _check(nch, chunk, nl, his, steps, calls, lookahead=2):
    kinds = [k for k, _ in steps]
    # every pass-A chunk once, in order; the exchange once, right after the last one; every pass-B chunk once
    assert [c for k, c in steps if k == "A"] == list(range(nch))
    assert kinds.count("exchange") == 1
    pos_x = kinds.index("exchange")
    assert steps[pos_x - 1] == ("A", nch - 1) or steps[pos_x - 1][0] == "B"
    assert all(k != "A" for k in kinds[pos_x:])
    b = [c for k, c in steps if k in ("B", "early_B")]
    assert sorted(b) == list(range(nch))
    pos_a = {c: i for i, (k, c) in enumerate(steps) if k == "A"}
    for i, (k, c) in enumerate(steps):
        if k not in ("B", "early_B"):
            continue
        hi = his[c]
        if hi >= nl:                                  # a ghost sender: only after the H1 exchange
            assert i > pos_x
        else:
            need = c if hi < 0 else max(c, hi // chunk)
            assert i > pos_a[need]                    # every chunk holding one of its senders is done
        if k == "early_B":
            assert i < pos_a[nch - 1]
    # the host asks for chunk c's range in order, and not before pass-A chunk c + lookahead - 1 was issued
    assert [c for c, _ in calls] == list(range(nch))
    for c, n_issued in calls:
        assert n_issued >= min(nch, c + lookahead)


def test_slab_order_interleaves_pass_b():
    """Chunks of z slabs: senders within the next three chunks, the first two chunks wrap around the periodic box."""
    nch, chunk = 40, 100
    nl = nch * chunk
    his = [nl - 1 if c < 2 else min((c + 3) * chunk - 1, nl - 1) for c in range(nch)]
    steps, calls = _run(nch, chunk, nl, his)
    _check(nch, chunk, nl, his, steps, calls)
    early = sum(k == "early_B" for k, _ in steps)
    assert early >= nch - 6                           # all but the wrapping and the last few start early


def test_ghost_chunks_wait_for_the_exchange_and_empty_chunks_run_at_once():
    nch, chunk = 12, 64
    nl = nch * chunk
    his = [nl + 5 if c in (0, 11) else -1 if c == 5 else min((c + 2) * chunk, nl - 1) for c in range(nch)]
    steps, calls = _run(nch, chunk, nl, his)
    _check(nch, chunk, nl, his, steps, calls)
    pos_x = [k for k, _ in steps].index("exchange")
    assert {c for k, c in steps[pos_x:] if k == "B"} >= {0, 11}
    assert ("early_B", 5) in steps


@pytest.mark.parametrize("lookahead", [1, 2, 4])
def test_random_sender_ranges(lookahead):
    rng = np.random.default_rng(3)
    for _ in range(20):
        nch = int(rng.integers(1, 30))
        chunk = int(rng.integers(1, 50))
        nl = nch * chunk - int(rng.integers(0, chunk))
        his = [int(x) for x in rng.integers(-1, nl + 3, size=nch)]
        steps, calls = _run(nch, chunk, max(nl, 1), his, lookahead)
        _check(nch, chunk, max(nl, 1), his, steps, calls, lookahead)


def test_sc_coef_layout():
    rng = np.random.default_rng(0)
    sc = rng.normal(size=(2, 10, 8))
    out = E.sc_coef_layout(sc)
    assert out.shape == (2, 3, 8, 4) and out.flags["C_CONTIGUOUS"]
    for s in range(2):
        for t in range(12):
            for c in range(8):
                want = sc[s, t, c] if t < 10 else 0.0
                assert out[s, t // 4, c, t % 4] == want


def test_lammps_bin_order():
    rng = np.random.default_rng(1)
    box = np.array([20.0, 14.0, 31.0])
    pos = rng.uniform(-5.0, 40.0, size=(3000, 3))            # outside the box too: wrapped like LAMMPS's atoms
    o = S.lammps_bin_order(pos, box, binsize=3.5)
    assert sorted(o.tolist()) == list(range(len(pos)))
    nb = np.floor(box / 3.5).astype(int)
    c = np.minimum((np.remainder(pos, box) / (box / nb)).astype(int), nb - 1)
    key = (c[:, 2] * nb[1] + c[:, 1]) * nb[0] + c[:, 0]
    k = key[o]
    assert (np.diff(k) >= 0).all()                             # bins x fastest, then y, then z
    same = np.diff(k) == 0
    assert (np.diff(o)[same] > 0).all()                        # stable inside a bin
