"""Golden vectors produced by the reference's own code for this path, run on the CPU with the oracle's block math.

    python tests/golden/make_reference_pins.py PATH/TO/mace-million

writes tests/golden/reference_pins.npz next to this script.  The reference package is imported from the given
checkout by tests/golden/ref_adapter.py (it is never copied); the model is the seed-0 random-init MACE of the other
fixtures with non-zero atomic energies and a non-zero shift, so that the E0 + shift bookkeeping is pinned as well.
The structure is the reference's own 192-atom water cell (tests/golden/water64_n192.npz).

Cases (reference code that ran, inputs, what is stored):
* ``mliap``: ThreePassMLIAP.compute_forces (mliap_threepass.py:444-616) with FastLayers (fast_layers.py:108-223),
  exact radial MLP (spline_grid=0; the spline kernels are Triton, GPU only), chunk 80 (a partial tail chunk),
  node_bucket 256 and e_align 1024 (padding edges and nodes present) on the minimum-image pair list, sorted:
  eatoms [192] and pair forces dE/drij [P, 3] (the reference accumulates them in fp32).
* ``ghost``: the same entry point with explicit ghost atoms (one per boundary-crossing pair, owner exchange through
  the ML-IAP callbacks) and the pair list in a seeded random order (the reference sorts and un-permutes), chunk 64.
* ``alloy``: the same entry point on a 16-element bcc alloy (5^3 cells, 250 atoms, 15 A box; the seed-1 model with
  seeded E0): FastLayers' SpeciesSkip over 16 species columns, per-species E0, chunk 96.
* ``rc``: ReceiverChunkMACE.compute (receiver_chunk_mace.py:260-388) on the reference's System (Morton order, its
  own cell-list neighbour list) with LocalGraph padding (pad=True), FastLayers installed as the reference's
  fast_layers.install does, chunk 64: total energy and atom forces (original atom order), and a checksum of its
  neighbour list's (receiver, sender) pairs in the original atom order.
* ``rc_ace``: the same ReceiverChunkMACE run with the reference's exact density-projection layer 1
  (ace_layer1.py:23-105, installed over FastLayers as ace_layer1.install does).  Its path table (fused_edge_conv.
  path_table reads it from cuEquivariance, absent here) is this build's layer-1 channelwise TP table, the same terms.
* ``tables``: conv_spline.build_tables (conv_spline.py:230-249) for species (H, O), 512 knots over [0.5, r_max]:
  knot rows 0, 1, 255, 510, 511 of TV and TG (fp32) of every ordered species pair, both interaction blocks.
* ``xchg``: mliap_threepass._exchange (mliap_threepass.py:40-55) on meta tensors (no memory) of ntotal x D arrays
  beyond 2^31 elements: the column width of each callback, in call order.
* ``hermite``: spline_radial._hermite_eval (spline_radial.py:37-57), value and d/dr, on fp64 tables of block 1 at
  radii below the first knot, inside, on knots and near r_max (first 64 columns).
"""
import dataclasses
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "mace-million_b200"), ROOT, HERE]

from mace_onegpu import model as M  # noqa: E402
from mace_onegpu import neighbors as NB  # noqa: E402
from mace_onegpu import structures as S  # noqa: E402
from mace_onegpu.mliap_data import MLIAPData  # noqa: E402
from oracle import mace_ref  # noqa: E402

import ref_adapter  # noqa: E402

E0_SEED, SHIFT = 7, 0.25
TABLE_ROWS = (0, 1, 255, 510, 511)
HERMITE_COLS = 64
XCHG_CASES = ((1000, 512), (4_194_304, 512), (9_000_000, 512), (5_000_000, 500), (7_000_000, 700),
              (1_000_000_000, 5), (2 ** 31, 3))


# ------------------------------------------------------------------------------------------ shared with the tests
def pin_model(seed=0):
    """The seed-`seed` model with seeded non-zero atomic energies and shift (a MACEModel, for the CUDA path too)."""
    base = M.default_model(seed)
    state = {k: v.clone() for k, v in base.params().items()}
    g = torch.Generator().manual_seed(E0_SEED)
    state["atomic_energies"] = -2.0 + torch.randn(state["atomic_energies"].shape, generator=g, dtype=torch.float64)
    return M.MACEModel(dataclasses.replace(base.arch, shift=SHIFT), state)


def cell():
    g = np.load(os.path.join(HERE, "water64_n192.npz"))
    return g["pos"], g["Z"], g["box"]


def pair_checksum(pi, pj):
    pi, pj = torch.as_tensor(pi).long(), torch.as_tensor(pj).long()
    w = torch.arange(1, pi.numel() + 1, dtype=torch.int64)
    return int(((pi * 1000003 + pj) * w).sum())


def inputs(mdl):
    """Minimum-image list, and the ghost / shuffled variant: (pi, pj, rij, cols, n), (pi, pj, rij, cols2, n, owner)."""
    pos, Z, box = cell()
    cols = torch.as_tensor(S.species_columns(Z, mdl.arch.atomic_numbers))
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    n = len(Z)
    d = torch.as_tensor(pos)[pi.long()] - torch.as_tensor(pos)[pj.long()]
    cross = (rij - d).abs().sum(1) > 1e-9
    ghosts = pj.long()[cross]
    pj2 = pj.clone()
    pj2[cross] = (n + torch.arange(int(cross.sum()))).to(pj.dtype)
    owner = torch.cat([torch.arange(n), ghosts])
    cols2 = torch.cat([cols, cols[ghosts]])
    perm = torch.randperm(pi.numel(), generator=torch.Generator().manual_seed(3))
    return (pi, pj, rij, cols, n), (pi[perm], pj2[perm], rij[perm], cols2, n, owner)


def alloy_inputs(mdl):
    """(pi, pj, rij, cols, n) of the 250-atom 16-element alloy, minimum image."""
    pos, Z, box = S.alloy_bcc(5, seed=0)
    cols = torch.as_tensor(S.species_columns(Z, mdl.arch.atomic_numbers))
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    return pi, pj, rij, cols, len(Z)


# ------------------------------------------------------------------------------------------ the reference runs
def _mliap(mod, model, data, chunk):
    """eatoms (fp64), pair forces (fp32: the reference sums them in fp32, so the cast is exact), energy."""
    tp = mod("mliap_threepass").ThreePassMLIAP(model, chunk=chunk, spline_grid=0, node_bucket=256, e_align=1024)
    tp.compute_forces(data)
    pf = torch.as_tensor(data.pair_forces)
    assert torch.equal(pf.float().double(), pf)
    return data.eatoms.clone(), pf.float().clone(), float(data.energy)


def main(ref_root):
    mdl = pin_model()
    arch = dataclasses.asdict(mdl.arch)
    ref = mace_ref.MaceRef(mdl.params(), arch)
    adapter = ref_adapter.OracleMACE(ref, mdl.arch.atomic_numbers)
    (pi, pj, rij, cols, n), (gpi, gpj, grij, gcols, _, owner) = inputs(mdl)
    out = dict(atomic_energies=mdl.p("atomic_energies").numpy(), shift=np.float64(SHIFT),
               n_pairs=np.int64(pi.numel()), pair_checksum=np.int64(pair_checksum(pi, pj)),
               ghost_checksum=np.int64(pair_checksum(gpi, gpj)), n_total_ghost=np.int64(gcols.numel()))
    with ref_adapter.reference_env(ref_root) as mod:
        eat, pf, energy = _mliap(mod, adapter, MLIAPData(pi, pj, rij, cols, n), 80)
        out.update(mliap_eat=eat.numpy(), mliap_pf=pf.numpy(), mliap_energy=np.float64(energy))
        eat, pf, energy = _mliap(mod, adapter, MLIAPData(gpi, gpj, grij, gcols, n, owner=owner), 64)
        out.update(ghost_eat=eat.numpy(), ghost_pf=pf.numpy(), ghost_energy=np.float64(energy))
        amdl = pin_model(1)
        aad = ref_adapter.OracleMACE(mace_ref.MaceRef(amdl.params(), dataclasses.asdict(amdl.arch)),
                                     amdl.arch.atomic_numbers)
        api, apj, arij, acols, an = alloy_inputs(amdl)
        eat, pf, energy = _mliap(mod, aad, MLIAPData(api, apj, arij, acols, an), 96)
        out.update(alloy_eat=eat.numpy(), alloy_pf=pf.numpy(), alloy_energy=np.float64(energy),
                   alloy_checksum=np.int64(pair_checksum(api, apj)), alloy_species=np.int64(torch.unique(acols).numel()))

        rc, fl = mod("receiver_chunk_mace"), mod("fast_layers")
        pos, Z, box = cell()
        sysm = rc.System(torch.as_tensor(pos, dtype=torch.float64), torch.as_tensor(box), cols.clone(),
                         float(mdl.arch.r_max), "cpu")
        sysm.build_neighbors()
        # its neighbour list (System.build_neighbors, receiver_chunk_mace.py:113-165) as (receiver, sender) pairs in
        # the original atom order, sorted like this build's host list
        rows = torch.repeat_interleave(torch.arange(sysm.N), sysm.NN.long())
        senders = sysm.NL.long()[sysm.NL >= 0]
        gi, gj = sysm.perm[rows], sysm.perm[senders]
        o = torch.argsort(gi * sysm.N + gj)
        out["rc_pair_checksum"] = np.int64(pair_checksum(gi[o], gj[o]))
        saved = rc.layer1, rc.layer2_energy
        try:
            fl.install(adapter, sorted(torch.unique(cols).tolist()))
            E, F, _t, _p = rc.ReceiverChunkMACE(adapter, torch.float64, 64, pad=True, node_bucket=256).compute(
                sysm, log=lambda *a: None)
        finally:
            rc.layer1, rc.layer2_energy = saved
        Fo = torch.empty_like(F)
        Fo[sysm.perm] = F
        out.update(rc_energy=np.float64(E), rc_F=Fo.numpy(), rc_n_pairs=np.int64(int(sysm.NN.sum())))

        fec, ace = mod("fused_edge_conv"), mod("ace_layer1")
        t1 = M.tp_tables()[0]
        table = dict(C=int(mdl.arch.channels), nW=t1["nW"], nX=t1["nX"], nY=t1["nY"], nO=t1["nO"],
                     terms=[(int(w), int(k), int(m), int(o), float(c)) for (w, k, m, o, c) in t1["terms"]])
        saved_table = fec.path_table
        fec.path_table = lambda block: table
        try:
            cs = sorted(torch.unique(cols).tolist())
            fl.install(adapter, cs)
            ace.install(adapter, cs)
            E, F, _t, _p = rc.ReceiverChunkMACE(adapter, torch.float64, 64, pad=True, node_bucket=256).compute(
                sysm, log=lambda *a: None)
        finally:
            rc.layer1, rc.layer2_energy = saved
            fec.path_table = saved_table
        Fo = torch.empty_like(F)
        Fo[sysm.perm] = F
        out.update(rc_ace_energy=np.float64(E), rc_ace_F=Fo.numpy())

        zs = [1, 8]
        tab = mod("conv_spline").build_tables(adapter, zs, n_grid=512, r_lo=0.5, device="cpu")
        M_ = tab["M"]
        rows = torch.as_tensor(TABLE_ROWS)
        for i, (TV, TG) in enumerate(tab["tables"]):
            P = TV.shape[0] // M_
            out[f"tab{i}_TV"] = TV.view(P, M_, -1)[:, rows].numpy()
            out[f"tab{i}_TG"] = TG.view(P, M_, -1)[:, rows].numpy()
        out.update(tab_r_lo=np.float64(tab["r_lo"]), tab_r_hi=np.float64(tab["r_hi"]), tab_M=np.int64(M_))

        xg = mod("mliap_threepass")._exchange
        for nt_, D_ in XCHG_CASES:
            widths = []
            xg(lambda s_, d_, w_: widths.append((s_.shape[1], w_)), torch.empty(nt_, D_, device="meta"),
               torch.empty(nt_, D_, device="meta"), D_)
            out[f"xchg_{nt_}_{D_}"] = np.array(widths, dtype=np.int64)

        sr = mod("spline_radial")
        t = mace_ref.MaceRef(mdl.params(), arch, spline_knots=512).tables[1]
        V, G = t["TV"][:, :HERMITE_COLS].contiguous(), t["TG"][:, :HERMITE_COLS].contiguous()
        h = t["h"]
        r = torch.cat([torch.tensor([0.18, 0.3, 0.49, 0.5, 0.5 + h, 0.5 + 255 * h, 6.0 - 2 * h, 6.0 - 1.01 * h]),
                       torch.linspace(0.55, 5.9, 41, dtype=torch.float64)]).to(torch.float64)
        pair = torch.zeros(r.numel(), dtype=torch.long)
        out.update(herm_r=r.numpy(),
                   herm_W=sr._hermite_eval(V, G, 512, 0.5, h, r, pair, False).numpy(),
                   herm_dW=sr._hermite_eval(V, G, 512, 0.5, h, r, pair, True).numpy())
    np.savez_compressed(os.path.join(HERE, "reference_pins.npz"), **out)
    print(f"mliap: E = {out['mliap_energy']:.6f} eV; ghost: E = {out['ghost_energy']:.6f} eV; "
          f"rc: E = {out['rc_energy']:.6f} eV ({int(out['rc_n_pairs'])} pairs)")


if __name__ == "__main__":
    main(sys.argv[1])
