"""The reference-facing plugin: ThreePassMLIAP.compute_forces(data) with an ML-IAP data object, on the GPU.

Device-resident inputs against the CPU fp64 oracle (the north_star tolerances); pinned host inputs and outputs (the
engine streams senders / vectors in chunk by chunk during pass A and hands every finished chunk's pair forces to
the host during pass C) against the device-resident call; the pipelined pass A / B schedule of a streamed pair list
against the serial one, without and with ghost atoms; shuffled host input (no overlap: the engine sorts);
a pickle round trip of the plugin object (LAMMPS unpickles it from the model file)."""
import dataclasses
import io

import pytest
import torch

from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import structures as S
from mace_onegpu.mliap_data import MLIAPData
from mace_onegpu.mliap_threepass import ThreePassMLIAP
from oracle import mace_ref

pytestmark = pytest.mark.gpu

E_TOL = 1e-5      # eV per atom
F_TOL = 1e-3      # eV / A


@pytest.fixture(scope="module")
def setup():
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, seed=0)
    cols = torch.as_tensor(S.species_columns(Z, mdl.arch.atomic_numbers))
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), spline_knots=512)
    eat, pf = ref.three_pass(pi, pj, rij, cols, len(Z), 64)
    return dict(mdl=mdl, n=len(Z), cols=cols, pi=pi, pj=pj, rij=rij, eat=eat, pf=pf)


def _device_data(s):
    d = "cuda"
    return MLIAPData(s["pi"].to(d), s["pj"].to(d), s["rij"].to(d), s["cols"].to(d), s["n"])


def _host_data(s, perm=None):
    pi, pj, rij = s["pi"], s["pj"], s["rij"]
    if perm is not None:
        pi, pj, rij = pi[perm], pj[perm], rij[perm]
    return MLIAPData(pi.contiguous().pin_memory(), pj.contiguous().pin_memory(), rij.contiguous().pin_memory(),
                     s["cols"].clone().pin_memory(), s["n"], host_outputs=True)


def test_device_inputs_match_oracle(setup):
    mli = ThreePassMLIAP(setup["mdl"], chunk=64)
    data = _device_data(setup)
    mli.compute_forces(data)
    torch.cuda.synchronize()
    assert (data.eatoms.cpu() - setup["eat"]).abs().max() < E_TOL
    assert abs(data.energy - float(setup["eat"].sum())) < E_TOL * setup["n"]
    assert (data.pair_forces.cpu() - setup["pf"]).abs().max() < F_TOL


def test_pinned_host_io_overlap_matches_device(setup):
    """Many chunks (chunk = 32 receivers): per-chunk H2D waits in pass A and per-chunk D2H hand-out in pass C."""
    mli = ThreePassMLIAP(setup["mdl"], chunk=32)
    dev = _device_data(setup)
    mli.compute_forces(dev)
    host = _host_data(setup)
    mli.compute_forces(host)
    assert mli._eng.host_pf_written
    torch.cuda.synchronize()
    assert host.pair_forces.data_ptr() == host.pair_forces_host.data_ptr()
    assert (host.eatoms - dev.eatoms.cpu()).abs().max() < 1e-9
    assert (host.pair_forces - dev.pair_forces.cpu()).abs().max() < 1e-5
    assert (host.pair_forces - setup["pf"]).abs().max() < F_TOL
    # a second call reuses the cached events and side stream
    mli.compute_forces(host)
    torch.cuda.synchronize()
    assert (host.pair_forces - setup["pf"]).abs().max() < F_TOL


def test_pipelined_schedule_matches_serial():
    """A streamed pair list of a box long in z, in LAMMPS's bin order (z slabs; 24 chunks of 32 receivers): pass-B
    chunks run interleaved with pass A as soon as their senders are covered.  Same energies and pair forces as the
    serial schedule; a Morton-ordered copy (wider sender ranges) has more chunks wait for late pass-A chunks."""
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, 4, 16, seed=3)
    for order in ("lammps", "morton"):
        o = S.lammps_bin_order(pos, box) if order == "lammps" else S.morton_order(pos, box)
        p, z = pos[o], Z[o]
        cols = torch.as_tensor(S.species_columns(z, mdl.arch.atomic_numbers))
        pi, pj, rij = NB.neighbor_list(p, box, mdl.arch.r_max)
        s = dict(pi=pi, pj=pj, rij=rij, cols=cols, n=len(z))
        mli = ThreePassMLIAP(mdl, chunk=32)
        pip = _host_data(s)
        mli.compute_forces(pip)                          # the engine's default schedule for this input
        assert mli._eng.last_schedule == "pipelined"
        if order == "lammps":
            assert mli._eng.early_b_chunks >= 12          # most chunks ran before pass A's last chunk
        mli._eng.pipeline = False
        ser = _host_data(s)
        mli.compute_forces(ser)
        assert mli._eng.last_schedule == "serial"
        torch.cuda.synchronize()
        for _ in range(2):
            assert (pip.eatoms - ser.eatoms).abs().max() < 1e-9
            assert (pip.pair_forces - ser.pair_forces).abs().max() < 1e-5 * ser.pair_forces.abs().max() + 1e-7
            mli._eng.pipeline = True                      # again, with the side stream and events reused
            mli.compute_forces(pip)
            assert mli._eng.last_schedule == "pipelined"
            torch.cuda.synchronize()


def test_pipelined_schedule_with_ghosts():
    """Streamed pair list with explicit ghost atoms (the periodic images across the z faces of a box long in z, in
    LAMMPS's bin order) and owner-map exchanges: the chunks in the middle of the box have no ghost sender and run
    during pass A, the end chunks after the H1 exchange.  Same results as the serial schedule and as the same box
    without ghosts (minimum image)."""
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, 4, 16, seed=4)
    o = S.lammps_bin_order(pos, box)
    pos, Z = pos[o], Z[o]
    n = len(Z)
    cols = torch.as_tensor(S.species_columns(Z, mdl.arch.atomic_numbers))
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    d = torch.as_tensor(pos)[pi.long()] - torch.as_tensor(pos)[pj.long()]
    cross = (rij[:, 2] - d[:, 2]).abs() > 1e-9                 # pairs across a z face: the sender is a ghost
    pj2 = pj.clone()
    pj2[cross] = n + torch.arange(int(cross.sum()), dtype=pj.dtype)
    owner = torch.cat([torch.arange(n), pj[cross].long()])
    cols2 = torch.cat([cols, cols[pj[cross].long()]])

    def ghost_data():
        return MLIAPData(pi.contiguous().pin_memory(), pj2.contiguous().pin_memory(), rij.contiguous().pin_memory(),
                         cols2.clone().pin_memory(), n, owner=owner, host_outputs=True)

    mli = ThreePassMLIAP(mdl, chunk=32)
    pip = ghost_data()
    mli.compute_forces(pip)
    assert mli._eng.last_schedule == "pipelined"
    assert mli._eng.early_b_chunks >= 8
    mli._eng.pipeline = False
    ser = ghost_data()
    mli.compute_forces(ser)
    assert mli._eng.last_schedule == "serial"
    plain = _host_data(dict(pi=pi, pj=pj, rij=rij, cols=cols, n=n))
    mli.compute_forces(plain)
    torch.cuda.synchronize()
    for other in (ser, plain):
        assert (pip.eatoms - other.eatoms).abs().max() < 1e-9
        assert (pip.pair_forces - other.pair_forces).abs().max() < 1e-5 * other.pair_forces.abs().max() + 1e-7


def test_shuffled_host_inputs(setup):
    g = torch.Generator().manual_seed(1)
    o = torch.randperm(setup["pi"].numel(), generator=g)
    mli = ThreePassMLIAP(setup["mdl"], chunk=64)
    host = _host_data(setup, o)
    mli.compute_forces(host)
    assert not mli._eng.host_pf_written          # unsorted input: copied, sorted, results copied at the end
    torch.cuda.synchronize()
    assert (host.eatoms - setup["eat"]).abs().max() < E_TOL
    assert (host.pair_forces - setup["pf"][o]).abs().max() < F_TOL


def test_pickle_round_trip(setup):
    mli = ThreePassMLIAP(setup["mdl"], chunk=64)
    mli.compute_forces(_device_data(setup))
    buf = io.BytesIO()
    torch.save(mli, buf)
    buf.seek(0)
    mli2 = torch.load(buf, weights_only=False)
    assert not hasattr(mli2, "_eng")              # runtime state is not pickled
    assert mli2.element_types == mli.element_types and mli2.rcutfac == mli.rcutfac
    data = _device_data(setup)
    mli2.compute_forces(data)
    torch.cuda.synchronize()
    assert (data.eatoms.cpu() - setup["eat"]).abs().max() < E_TOL
