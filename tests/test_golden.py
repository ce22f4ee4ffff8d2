"""Golden vectors on the reference's own 192-atom water structure (examples/data/water64_1x1x1_N192.data of the
reference, read by tests/golden/make_water64.py into tests/golden/water64_n192.npz together with the fp64 oracle's
energies and forces for the seed-0 random-init model).

CPU: the fixture is the reference's cell (64 O + 128 H, 12.4138 A box), the oracle still reproduces the stored values
(regression pin), and its 512-knot tables stay within the force tolerance of the exact radial MLP on this structure.
GPU: the CUDA path, in both layer-1 forms and both GEMM paths, matches the stored spline values within the north_star
tolerances (1e-5 eV per atom, 1e-3 eV/A)."""
import dataclasses
import os

import numpy as np
import pytest
import torch

from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import structures as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "water64_n192.npz")
E_TOL = 1e-5      # eV per atom
F_TOL = 1e-3      # eV / A


@pytest.fixture(scope="module")
def golden():
    g = dict(np.load(GOLDEN))
    mdl = M.default_model(0)
    cols = S.species_columns(g["Z"], mdl.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(g["pos"], g["box"], mdl.arch.r_max)
    return dict(g, mdl=mdl, cols=cols, pi=pi, pj=pj, rij=rij, n=len(g["Z"]))


def test_fixture_is_the_reference_cell(golden):
    assert golden["n"] == 192 and (golden["Z"] == 8).sum() == 64 and (golden["Z"] == 1).sum() == 128
    assert np.allclose(golden["box"], 12.4138)
    assert golden["pi"].numel() == int(golden["n_pairs"])
    # every O has two H within 1.1 A (intact molecules)
    pos, box = golden["pos"], golden["box"]
    d = pos[golden["Z"] == 8][:, None, :] - pos[golden["Z"] == 1][None, :, :]
    d -= box * np.round(d / box)
    assert ((np.linalg.norm(d, axis=2) < 1.1).sum(1) == 2).all()


def test_oracle_reproduces_golden(golden):
    from oracle import mace_ref

    ref = mace_ref.MaceRef(golden["mdl"].params(), dataclasses.asdict(golden["mdl"].arch), spline_knots=512)
    eat, pf = ref.three_pass(golden["pi"], golden["pj"], golden["rij"], golden["cols"], golden["n"], 64)
    F = mace_ref.atom_forces(golden["pi"], golden["pj"], pf, golden["n"]).numpy()
    assert np.abs(eat.numpy() - golden["eat_spline512"]).max() < 1e-10
    assert np.abs(F - golden["F_spline512"]).max() < 1e-10
    assert np.abs(golden["F_spline512"].sum(0)).max() < 1e-9                    # no net force
    # the 512-knot tables against the exact radial MLP on the same structure
    assert np.abs(golden["eat_spline512"] - golden["eat_exact"]).max() < E_TOL
    assert np.abs(golden["F_spline512"] - golden["F_exact"]).max() < F_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("use_tc", [True, False], ids=["tcgen05", "simt"])
@pytest.mark.parametrize("l1_mode", ["density", "direct"])
def test_cuda_path_matches_golden(golden, use_tc, l1_mode):
    from mace_onegpu import engine as E
    from oracle import mace_ref

    eng = E.ThreePassEngine(golden["mdl"], sorted(set(golden["cols"].tolist())), chunk=64, device="cuda",
                            use_tc=use_tc, l1_mode=l1_mode)
    plan = eng.plan(golden["pi"], golden["pj"], golden["rij"], torch.as_tensor(golden["cols"]), golden["n"],
                    golden["n"])
    eat, pf = eng.evaluate(plan)
    torch.cuda.synchronize()
    F = mace_ref.atom_forces(golden["pi"], golden["pj"], pf.cpu(), golden["n"]).numpy()
    de = np.abs(eat.cpu().numpy() - golden["eat_spline512"]).max()
    dF = np.abs(F - golden["F_spline512"]).max()
    print(f"golden water64 ({l1_mode}, {'tcgen05' if use_tc else 'simt'}): max|dE_i| {de:.2e} eV, max|dF| {dF:.2e} eV/A")
    assert de < E_TOL and dF < F_TOL
