"""Error paths of the force evaluation, each driven by host-side injection (no GPU fault is involved: the kernels check
their inputs, record a bit in the status word and skip the bad edge; the host turns the word into a RuntimeError).

* non-finite and zero-length edge vectors -> "non-finite or zero edge vector";
* pair_i disagreeing with its CSR row (a corrupted plan) -> "pair_i does not match its CSR row";
* a sender index outside [0, ntotal) -> "sender index out of range";
* the force guard of the ML-IAP wrapper (mliap_threepass.py:595-601 in the reference): MACE3P_FMAX_ABORT below the
  largest pair force -> RuntimeError before LAMMPS would integrate the forces.
After every failure the same engine evaluates a clean input correctly (the context stays usable)."""
import dataclasses

import pytest
import torch

from mace_onegpu import engine as E
from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import structures as S
from mace_onegpu.mliap_data import MLIAPData
from mace_onegpu.mliap_threepass import ThreePassMLIAP
from oracle import mace_ref

pytestmark = pytest.mark.gpu

E_TOL = 1e-5
F_TOL = 1e-3


@pytest.fixture(scope="module")
def s():
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, seed=0)
    cols = torch.as_tensor(S.species_columns(Z, mdl.arch.atomic_numbers))
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), spline_knots=512)
    eat, pf = ref.three_pass(pi, pj, rij, cols, len(Z), 64)
    eng = E.ThreePassEngine(mdl, sorted(set(cols.tolist())), chunk=64, device="cuda")
    return dict(mdl=mdl, n=len(Z), cols=cols, pi=pi, pj=pj, rij=rij, eat=eat, pf=pf, eng=eng)


def _clean_run_still_correct(s):
    eng = s["eng"]
    plan = eng.plan(s["pi"], s["pj"], s["rij"], s["cols"].cuda(), s["n"], s["n"])
    eat, pf = eng.evaluate(plan)
    torch.cuda.synchronize()
    assert (eat.cpu() - s["eat"]).abs().max() < E_TOL
    assert (pf.cpu() - s["pf"]).abs().max() < F_TOL


def _expect(s, pi, pj, rij, msg, corrupt=None):
    eng = s["eng"]
    plan = eng.plan(pi, pj, rij, s["cols"].cuda(), s["n"], s["n"])
    if corrupt is not None:
        corrupt(plan)
    with pytest.raises(RuntimeError, match=msg):
        eng.evaluate(plan)
    _clean_run_still_correct(s)


@pytest.mark.parametrize("bad", [float("nan"), float("inf"), 0.0], ids=["nan", "inf", "zero"])
def test_nonfinite_or_zero_edge_vector(s, bad):
    rij = s["rij"].clone()
    rij[s["pi"].numel() // 2] = bad
    _expect(s, s["pi"], s["pj"], rij, "non-finite or zero edge vector")


def test_pair_i_disagrees_with_csr_row(s):
    def corrupt(plan):
        e = int(plan.rowptr[10].item()) + 3           # an edge inside receiver 10's row now claims receiver 11
        plan.pi[e] = 11
    _expect(s, s["pi"], s["pj"], s["rij"], "pair_i does not match its CSR row", corrupt)


def test_sender_out_of_range(s):
    pj = s["pj"].clone()
    pj[7] = s["n"] + 5
    _expect(s, s["pi"], pj, s["rij"], "sender index out of range")


def test_force_guard(s, monkeypatch):
    monkeypatch.setenv("MACE3P_FMAX_ABORT", "1e-3")     # far below this model's largest pair force
    mli = ThreePassMLIAP(s["mdl"], chunk=64)
    data = MLIAPData(s["pi"].cuda(), s["pj"].cuda(), s["rij"].cuda(), s["cols"].cuda(), s["n"])
    with pytest.raises(RuntimeError, match="non-finite or absurd output"):
        mli.compute_forces(data)
    monkeypatch.delenv("MACE3P_FMAX_ABORT")
    mli2 = ThreePassMLIAP(s["mdl"], chunk=64)
    mli2.compute_forces(data)
    torch.cuda.synchronize()
    assert (data.eatoms.cpu() - s["eat"]).abs().max() < E_TOL
