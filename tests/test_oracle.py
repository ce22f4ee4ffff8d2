"""The CPU fp64 oracle pinned by the invariants the reference's own tests check (tests/gpu/test_threepass.py of
the reference: three-pass == full graph, chunk invariance, periodic replica) plus rotation / inversion invariance,
finite differences, zero net force, ghost exchange and the spline-table error.  Also: the product's O(3) constants
equal the oracle's independently computed ones."""
import dataclasses

import numpy as np
import pytest
import torch

from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import o3
from mace_onegpu import structures as S
from oracle import mace_ref, o3_ref

torch.set_num_threads(8)


@pytest.fixture(scope="module")
def mdl():
    return M.default_model(0)


@pytest.fixture(scope="module")
def ref(mdl):
    return mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch))


@pytest.fixture(scope="module")
def water(mdl):
    pos, Z, box = S.water_box(4, seed=0)
    spec = S.species_columns(Z, mdl.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    return dict(pos=pos, Z=Z, box=box, spec=spec, pi=pi, pj=pj, rij=rij, n=len(Z))


@pytest.fixture(scope="module")
def base(ref, water):
    return ref.three_pass(water["pi"], water["pj"], water["rij"], water["spec"], water["n"], 64)


def test_o3_constants_match_oracle():
    for l1 in range(4):
        for l2 in range(4):
            for l3 in range(abs(l1 - l2), min(l1 + l2, 3) + 1):
                assert np.abs(o3.wigner_3j(l1, l2, l3) - o3_ref.w3j(l1, l2, l3)).max() < 1e-10
    for L in (0, 1):
        for nu in (1, 2, 3):
            assert np.abs(o3.sc_U(nu, L) - o3_ref.U(nu, L)).max() < 1e-10
    u = np.random.default_rng(0).normal(size=(50, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    Y = o3.sh_np(3, u)
    Yr = np.concatenate([o3_ref.sh_real(l, u) for l in range(4)], 1)
    assert np.abs(Y - Yr).max() < 1e-12
    Yt = mace_ref.sh_torch(torch.as_tensor(u * 2.5)).numpy()
    assert np.abs(Y - Yt).max() < 1e-12


def test_tp_tables_counts():
    t1, t2 = M.tp_tables()
    assert (t1["nW"], t1["nX"], t1["nY"], t1["nO"], len(t1["terms"])) == (4, 1, 16, 16, 16)
    assert (t2["nW"], t2["nX"], t2["nY"], t2["nO"], len(t2["terms"])) == (10, 4, 16, 40, 86)


def test_three_pass_matches_full_graph(ref, water, base):
    e_fg, pf_fg = ref.full_graph(water["pi"], water["pj"], water["rij"], water["spec"], water["n"])
    e3, pf3 = base
    assert (e3 - e_fg).abs().max() < 1e-9
    assert (pf3 - pf_fg).abs().max() < 1e-9
    F = mace_ref.atom_forces(water["pi"], water["pj"], pf3, water["n"])
    assert F.abs().max() > 0.1                       # forces are O(1 eV/A), so absolute tolerances mean something
    assert F.sum(0).abs().max() < 1e-10


def test_chunk_invariance(ref, water, base):
    e1, pf1 = ref.three_pass(water["pi"], water["pj"], water["rij"], water["spec"], water["n"], 48)
    e2, pf2 = base
    assert (e1 - e2).abs().max() < 1e-10
    assert (pf1 - pf2).abs().max() < 1e-10


def test_rotation_and_inversion(ref, water, base):
    rng = np.random.default_rng(3)
    R = torch.as_tensor(o3._random_rotation(rng))
    rij = water["rij"]
    e, pf = base
    er, pfr = ref.three_pass(water["pi"], water["pj"], rij @ R.T, water["spec"], water["n"], 96)
    assert (er - e).abs().max() < 1e-10
    assert (pfr - pf @ R.T).abs().max() < 1e-10
    ei, pfi = ref.three_pass(water["pi"], water["pj"], -rij, water["spec"], water["n"], 96)
    assert (ei - e).abs().max() < 1e-10
    assert (pfi + pf).abs().max() < 1e-10


def test_finite_differences(ref, water, base):
    e, pf = base
    rij = water["rij"].clone()
    h = 1e-5
    for k, c in ((17, 0), (901, 1), (5000, 2)):
        if True:
            rp, rm = rij.clone(), rij.clone()
            rp[k, c] += h
            rm[k, c] -= h
            ep, _ = ref.full_graph(water["pi"], water["pj"], rp, water["spec"], water["n"])
            em, _ = ref.full_graph(water["pi"], water["pj"], rm, water["spec"], water["n"])
            fd = float((ep.sum() - em.sum()) / (2 * h))
            assert abs(fd - float(pf[k, c])) < 1e-6 * max(1.0, abs(fd))


def test_ghost_exchange(ref, mdl, water, base):
    """Explicit ghost atoms (periodic images of locals beyond the box face) reproduce minimum image."""
    pos, box, n = water["pos"], water["box"], water["n"]
    pi, pj, rij = water["pi"].long(), water["pj"].long(), water["rij"]
    # every pair whose image crosses the boundary gets a ghost copy of the sender
    d = torch.as_tensor(pos)[pi] - torch.as_tensor(pos)[pj]
    shift = (rij - d)
    cross = shift.abs().sum(1) > 1e-9
    ghosts = pj[cross]
    gidx = n + torch.arange(int(cross.sum()))
    pj2 = pj.clone()
    pj2[cross] = gidx
    owner = torch.cat([torch.arange(n), ghosts])
    spec2 = np.concatenate([water["spec"], water["spec"][ghosts.numpy()]])
    e, pf = ref.three_pass(pi, pj2, rij, spec2, n, 64, owner=owner)
    e0, pf0 = base
    assert (e - e0).abs().max() < 1e-10
    assert (pf - pf0).abs().max() < 1e-10


def test_spline_tables_close_to_exact(mdl, water, base):
    refs = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), spline_knots=512)
    e, pf = refs.three_pass(water["pi"], water["pj"], water["rij"], water["spec"], water["n"], 192)
    e0, pf0 = base
    F = mace_ref.atom_forces(water["pi"], water["pj"], pf, water["n"])
    F0 = mace_ref.atom_forces(water["pi"], water["pj"], pf0, water["n"])
    assert (e - e0).abs().max() < 1e-5
    assert (F - F0).abs().max() < 1e-3
