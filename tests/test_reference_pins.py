"""The oracle, and through it the CUDA path, pinned against outputs of the reference's own code.

tests/golden/make_reference_pins.py ran the reference's ThreePassMLIAP.compute_forces (mliap_threepass.py:444-616,
FastLayers of fast_layers.py:108-223), ReceiverChunkMACE (receiver_chunk_mace.py:260-388), conv_spline.build_tables
(conv_spline.py:230-249) and spline_radial._hermite_eval (spline_radial.py:37-57) on the CPU, with the oracle's block
math behind mace-torch's module interface (tests/golden/ref_adapter.py), on the reference's 192-atom water cell, and
stored their outputs in tests/golden/reference_pins.npz.  The model is the seed-0 MACE with seeded atomic energies
and shift 0.25; the ML-IAP entry point also ran on a 250-atom 16-element alloy (seed-1 model, 16 species columns in
FastLayers' SpeciesSkip).

CPU: the oracle's own three-pass reproduces those outputs: per-atom energies to 1e-12 eV, pair forces to 1e-6 eV/A
(the reference accumulates pair forces in fp32; measured 5.3e-8), the receiver-chunk runs' total energy to 1e-9 eV
and atom forces to 1e-10 eV/A (with FastLayers, and with the reference's exact density-projection layer 1), the tables bit for bit (fp32) and the Hermite lookup and its derivative to 1e-10.
GPU: the CUDA path (512-knot tables) through ThreePassMLIAP.compute_forces reproduces the reference's ML-IAP outputs
(exact radial MLP) within the north_star tolerances, 1e-5 eV per atom and 1e-3 eV/A per pair force, without and with
ghost atoms and a shuffled pair list, and on the 16-element alloy (direct layer-1 form, per-species GEMM problems)."""
import dataclasses
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_reference_pins as R  # noqa: E402

E_TOL = 1e-5      # eV per atom (CUDA vs reference)
F_TOL = 1e-3      # eV / A (CUDA vs reference)


@pytest.fixture(scope="module")
def pins():
    g = dict(np.load(os.path.join(HERE, "golden", "reference_pins.npz")))
    mdl = R.pin_model()
    mliap, ghost = R.inputs(mdl)
    amdl = R.pin_model(1)
    return dict(g=g, mdl=mdl, mliap=mliap, ghost=ghost, amdl=amdl, alloy=R.alloy_inputs(amdl))


@pytest.fixture(scope="module")
def oracle_runs(pins):
    from oracle import mace_ref

    mdl = pins["mdl"]
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch))
    pi, pj, rij, cols, n = pins["mliap"]
    gpi, gpj, grij, gcols, _, owner = pins["ghost"]
    amdl = pins["amdl"]
    aref = mace_ref.MaceRef(amdl.params(), dataclasses.asdict(amdl.arch))
    return dict(mliap=ref.three_pass(pi, pj, rij, cols, n, 64),
                ghost=ref.three_pass(gpi, gpj, grij, gcols, n, 64, owner=owner),
                alloy=aref.three_pass(*pins["alloy"], 64))


def test_fixture_inputs_reproduced(pins):
    """The model and the pair lists the tests rebuild are the ones the reference ran on."""
    g = pins["g"]
    assert np.array_equal(pins["mdl"].p("atomic_energies").numpy(), g["atomic_energies"])
    pi, pj = pins["mliap"][:2]
    gpi, gpj, _, gcols = pins["ghost"][:4]
    assert pi.numel() == int(g["n_pairs"]) == int(g["rc_n_pairs"])
    assert R.pair_checksum(pi, pj) == int(g["pair_checksum"])
    # this build's host neighbour list has exactly the pairs of the reference's System.build_neighbors
    assert R.pair_checksum(pi, pj) == int(g["rc_pair_checksum"])
    assert R.pair_checksum(gpi, gpj) == int(g["ghost_checksum"]) and gcols.numel() == int(g["n_total_ghost"])
    api, apj, _, acols, _ = pins["alloy"]
    assert R.pair_checksum(api, apj) == int(g["alloy_checksum"])
    assert torch.unique(acols).numel() == int(g["alloy_species"]) == 16


@pytest.mark.parametrize("case", ["mliap", "ghost", "alloy"])
def test_oracle_matches_reference_mliap(pins, oracle_runs, case):
    g = pins["g"]
    eat, pf = oracle_runs[case]
    assert np.abs(eat.numpy() - g[f"{case}_eat"]).max() < 1e-12
    assert abs(float(eat.sum()) - float(g[f"{case}_energy"])) < 1e-10
    assert np.abs(pf.numpy() - g[f"{case}_pf"]).max() < 1e-6


@pytest.mark.parametrize("run", ["rc", "rc_ace"])
def test_oracle_matches_reference_receiver_chunk(pins, oracle_runs, run):
    """ReceiverChunkMACE with FastLayers ("rc") and with the reference's exact density-projection layer 1 installed
    over it ("rc_ace", ace_layer1.py): the same energy and atom forces as the oracle's standard three-pass."""
    from oracle import mace_ref

    g = pins["g"]
    pi, pj, _, _, n = pins["mliap"]
    eat, pf = oracle_runs["mliap"]
    F = mace_ref.atom_forces(pi, pj, pf, n).numpy()
    assert abs(float(eat.sum()) - float(g[f"{run}_energy"])) < 1e-9
    assert np.abs(F - g[f"{run}_F"]).max() < 1e-10


def test_oracle_tables_match_reference_build_tables(pins):
    """fp64 samples, central-difference slopes times h, every ordered species pair the same table, cast to fp32."""
    from oracle import mace_ref

    g, mdl = pins["g"], pins["mdl"]
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), spline_knots=int(g["tab_M"]))
    assert float(g["tab_r_lo"]) == ref.r_lo and float(g["tab_r_hi"]) == ref.rmax
    rows = list(R.TABLE_ROWS)
    for i in (0, 1):
        t = ref.tables[i]
        assert g[f"tab{i}_TV"].shape[0] == 4                                   # (H, O) x (H, O)
        assert np.array_equal(g[f"tab{i}_TV"], np.broadcast_to(t["TV"][rows].float().numpy(), g[f"tab{i}_TV"].shape))
        assert np.array_equal(g[f"tab{i}_TG"], np.broadcast_to(t["TG"][rows].float().numpy(), g[f"tab{i}_TG"].shape))


def test_oracle_hermite_matches_reference(pins):
    """Value and d/dr of the cubic Hermite lookup, also below the first knot (clamped, slope passed through)."""
    from oracle import mace_ref

    g, mdl = pins["g"], pins["mdl"]
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), spline_knots=512)
    r = torch.as_tensor(g["herm_r"]).clone().requires_grad_(True)
    W = ref.tp_weights(1, r.unsqueeze(-1), None)[:, :R.HERMITE_COLS]
    assert np.abs(W.detach().numpy() - g["herm_W"]).max() < 1e-10
    dW = torch.stack([torch.autograd.grad(W[:, c].sum(), r, retain_graph=True)[0] for c in range(W.shape[1])], 1)
    assert np.abs(dW.numpy() - g["herm_dW"]).max() < 1e-10


@pytest.mark.parametrize("nt,D", R.XCHG_CASES)
def test_exchange_split_matches_reference(pins, nt, D):
    """The callbacks of one exchange: the same column widths in the same order as the reference's _exchange, so
    that every LAMMPS comm buffer stays below 2^31 elements (meta tensors: sizes only, no memory)."""
    from mace_onegpu.mliap_threepass import _exchange, exchange_blocks

    calls = []
    _exchange(lambda s, d, w: calls.append((s.shape[1], w)), torch.empty(nt, D, device="meta"),
              torch.empty(nt, D, device="meta"), D)
    assert np.array_equal(np.array(calls, dtype=np.int64), pins["g"][f"xchg_{nt}_{D}"])
    blocks = exchange_blocks(nt, D)
    assert [w for _, w in blocks] == [w for _, w in calls]
    assert blocks[0][0] == 0 and all(b[0] + b[1] == c[0] for b, c in zip(blocks, blocks[1:]))
    assert blocks[-1][0] + blocks[-1][1] == D
    assert all(nt * w < 2 ** 31 - 1 or w == 1 for _, w in blocks)


def test_exchange_blocks_properties():
    """For any size: the blocks tile the columns in order, all but the last have the same width D >> k, k is the
    smallest shift for which a block stays below 2^31 - 1 elements (or the width is one column)."""
    from mace_onegpu.mliap_threepass import exchange_blocks

    rng = np.random.default_rng(5)
    for _ in range(2000):
        nt = int(rng.integers(1, 2 ** 33))
        D = int(rng.integers(1, 2049))
        blocks = exchange_blocks(nt, D)
        w = blocks[0][1]
        assert [c0 for c0, _ in blocks] == list(range(0, D, w))
        assert all(bw == w for _, bw in blocks[:-1]) and 0 < blocks[-1][1] <= w
        assert sum(bw for _, bw in blocks) == D
        assert nt * w < 2 ** 31 - 1 or w == 1
        k = next(k for k in range(64) if (D >> k) == w)
        assert k == 0 or (nt * (D >> (k - 1)) >= 2 ** 31 - 1 and (D >> (k - 1)) > 1)


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["mliap", "ghost", "alloy"])
def test_cuda_matches_reference_mliap(pins, case):
    from mace_onegpu.mliap_data import MLIAPData
    from mace_onegpu.mliap_threepass import ThreePassMLIAP

    g = pins["g"]
    d = "cuda"
    if case == "ghost":
        pi, pj, rij, cols, n, owner = pins["ghost"]
        data = MLIAPData(pi.to(d), pj.to(d), rij.to(d), cols.to(d), n, owner=owner)
    else:
        pi, pj, rij, cols, n = pins[case]
        data = MLIAPData(pi.to(d), pj.to(d), rij.to(d), cols.to(d), n)
    mli = ThreePassMLIAP(pins["amdl" if case == "alloy" else "mdl"], chunk=64)
    mli.compute_forces(data)
    torch.cuda.synchronize()
    assert np.abs(data.eatoms.cpu().numpy() - g[f"{case}_eat"]).max() < E_TOL
    assert abs(data.energy - float(g[f"{case}_energy"])) < E_TOL * n
    assert np.abs(torch.as_tensor(data.pair_forces).cpu().numpy() - g[f"{case}_pf"]).max() < F_TOL
