"""Multi-GPU MD driver logic on the CPU (gloo, world sizes 2, 4 and 8 on the bench's grids): md.DomainVelocityVerlet
against the single-process md.VelocityVerlet on the same periodic box.

The force provider is a stand-in with the ThreePassEngine calls the drivers use (plan / evaluate, with or without a
halo): a smooth pair potential phi(r) = eps (1 - r / rc)^4 on the given pair list, per-atom energy 1/2 sum phi over
the atom's pairs, pair forces dE/drij.  With a halo it also runs the forward and reverse exchanges of a per-atom row
holding the atom's global index, and asserts that every ghost row received its owner's index, so the exchange maps
of each rebuild are checked too.  Hot velocities and a 1 A skin force several decomposition / Verlet-list rebuilds
within the run; positions, velocities and energies must agree to fp64 round-off."""
import os
import socket
import sys
import types

import numpy as np
import pytest
import torch

from mace_onegpu import structures as S

R_MAX, SKIN, EPS = 4.0, 1.0, 0.05
STEPS = 14


class PairEngine:
    def __init__(self, device="cpu"):
        self.device = torch.device(device)
        self.model = types.SimpleNamespace(r_max=R_MAX)
        self.gid = None                      # global ids of the local + ghost rows (domain runs)

    def plan(self, pi, pj, rij, elems, nl, nt):
        return types.SimpleNamespace(pi=pi.long(), pj=pj.long(), rij=rij, nl=nl, nt=nt)

    def evaluate(self, plan, forward_exchange=None, reverse_exchange=None, halo=None):
        if halo is not None:
            forward_exchange, reverse_exchange = halo.forward, halo.reverse
        if forward_exchange is not None:
            H = torch.zeros(plan.nt, 2, dtype=torch.float64)
            H[:plan.nl, 0] = self.gid[:plan.nl].double()
            forward_exchange(H)
            assert torch.equal(H[plan.nl:, 0], self.gid[plan.nl:].double()), "ghost rows must hold their owners' rows"
            reverse_exchange(H)
        r = plan.rij.norm(dim=1)
        u = 1.0 - r / R_MAX
        eat = torch.zeros(plan.nl, dtype=torch.float64).index_add_(0, plan.pi, 0.5 * EPS * u ** 4)
        dphi = -4.0 * EPS * u ** 3 / R_MAX
        pf = (0.5 * dphi / r).unsqueeze(1) * plan.rij
        return eat, pf


def _system():
    pos, Z, box = S.water_box(9, 6, 6, seed=4)              # 27.9 x 18.6 x 18.6 A, 972 atoms
    vel = S.maxwell_boltzmann(Z, 3000.0, seed=2)
    cols = np.zeros(len(Z), dtype=np.int64)
    return pos, Z, box, vel, cols


def _single():
    from mace_onegpu.md import VelocityVerlet

    pos, Z, box, vel, cols = _system()
    md = VelocityVerlet(PairEngine(), pos, box, cols, Z, vel, dt=2.0, skin=SKIN)
    E = [md.epot]
    for _ in range(STEPS):
        md.step()
        E.append(md.epot)
    return md.x.numpy(), md.v.numpy(), np.array(E), md.rebuilds


def _worker(rank, world, port, grid, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from mace_onegpu.md import DomainVelocityVerlet

    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pos, Z, box, vel, cols = _system()
        eng = PairEngine()

        class Tracked(DomainVelocityVerlet):
            def _build(self):
                super()._build()
                eng.gid = self.gid

        md = Tracked(eng, pos, box, cols, Z, vel, grid, rank, dt=2.0, skin=SKIN)
        E = [md.epot]
        for _ in range(STEPS):
            md.step()
            E.append(md.epot)
        q.put((rank, md.x.numpy(), md.v.numpy(), np.array(E), md.rebuilds, md.nl))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def single():
    return _single()


@pytest.mark.parametrize("grid", [(2, 1, 1), (2, 2, 1), (2, 2, 2)], ids=["2-ranks", "4-ranks", "8-ranks"])
def test_domain_md_matches_single_process(single, grid):
    """The 2, 4 and 8-rank grids of the multi-GPU bench (2x1x1, 2x2x1, 2x2x2)."""
    import torch.multiprocessing as mp

    x1, v1, E1, nb1 = single
    world = int(np.prod(grid))
    assert nb1 >= 3                                          # the run crosses several rebuilds
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, grid, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue
    import time

    out, t0 = [], time.time()
    while len(out) < world:
        try:
            out.append(q.get(timeout=2))
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead and time.time() - t0 < 300, f"rank failed: exit codes {dead}"
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    out.sort(key=lambda t: t[0])
    n = x1.shape[0]
    assert sum(o[5] for o in out) == n                        # every atom owned by exactly one rank
    for rank, x, v, E, nb, nl in out:
        assert nb == nb1
        assert np.abs(x - x1).max() < 1e-9 and np.abs(v - v1).max() < 1e-9
        assert np.abs(E - E1).max() < 1e-9 * max(1.0, np.abs(E1).max())
    assert all(np.array_equal(out[0][1], o[1]) for o in out)  # replicated positions identical on every rank


if __name__ == "__main__":
    sys.exit(pytest.main([__file__, "-q"]))
