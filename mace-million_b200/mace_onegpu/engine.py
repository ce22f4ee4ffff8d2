"""Host side of the B200 three-pass force evaluation: folds the fp64 model into device buffers (mb_model_t), builds
the per-call plan (receiver CSR, species-sorted chunk order) and runs the native passes (mb_eval_t) with the H1
forward / G1 reverse halo exchanges between them.

Folding (exact algebra, fp64 on the host, then fp32 on the device):
* radial MLP constants folded into the matrices as in the reference's fused_radial.py:4-9
  (A0 = W0/sqrt(8), A_k = cst W_k / sqrt(64));
* layer-1 sender features X1 = linear_up(embedding(species)) depend only on the sender species, so they are folded
  into the layer-1 spline table (T1 = W1 * X1[s_send]; the exactness argument of the reference's ace_layer1.py:2-16);
* linear_1 and the species skip_tp of layer 1 commute with the per-receiver 1 / (rho + 1) and are folded into one
  per-species, per-l matrix M0[s][l];
* the symmetric contractions become per-(species, channel) monomial coefficients (o3.sc_entries order);
* e3nn's 1 / sqrt(fan_in) and normalize2mom constants are folded into every matrix.
"""
from __future__ import annotations

import heapq
import math
import os

import numpy as np
import torch

from . import _native as N
from . import model as Mdl
from . import o3

C = 128


def _f32(t, device):
    return torch.as_tensor(t, dtype=torch.float64).to(dtype=torch.float32, device=device).contiguous()


def tf32_rna(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to tf32 (10 mantissa bits), to nearest with ties away from zero (PTX cvt.rna.tf32.f32)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b & 0x7FFFFFFF) + np.uint32(0x1000)) & np.uint32(0x7FFFE000)
    r = r | (b & np.uint32(0x80000000))
    finite = (b & 0x7F800000) != 0x7F800000
    return np.where(finite, r, b).view(np.float32)


def tc_split(B: np.ndarray) -> np.ndarray:
    """K-major 3xTF32 planes of matrices B [..., K, N] used as GEMM B operands: [2][..., N, K] (hi, lo)."""
    bt = np.ascontiguousarray(np.swapaxes(np.asarray(B, dtype=np.float64), -1, -2)).astype(np.float32)
    hi = tf32_rna(bt)
    lo = tf32_rna(bt - hi)
    return np.ascontiguousarray(np.stack([hi, lo]))


def sw128_positions() -> np.ndarray:
    """Position of element (n, k) of a 128 x 128 K-major tile set in its shared-memory image: four K blocks of 32
    (16 KB each), each in the SWIZZLE_128B layout that tcgen05 descriptors read (8-row groups of 1024 B, row n at
    (n % 8) * 128 B, 16-byte chunk c of the row at chunk position c ^ (n % 8)).  Flat [n * 128 + k] -> float index."""
    n = np.arange(128)[:, None]
    k = np.arange(128)[None, :]
    c = (k % 32) // 4
    pos = (k // 32) * 4096 + (n // 8) * 256 + (n % 8) * 32 + (c ^ (n % 8)) * 4 + k % 4
    return pos.ravel()


def tc_planes(B: np.ndarray) -> np.ndarray:
    """GEMM B operands for the tcgen05 kernel: tf32 hi / lo planes (tc_split) with every 128 x 128 matrix permuted
    into its SWIZZLE_128B K-block image, so the kernel stages each 16 KB K block with one bulk copy.  Same shape,
    element count and matrix offsets as tc_split."""
    planes = tc_split(B)
    if planes.shape[-2:] != (128, 128):
        raise ValueError("tcgen05 GEMM operands are 128 x 128 matrices")
    flat = planes.reshape(-1, 128 * 128)
    out = np.empty_like(flat)
    out[:, sw128_positions()] = flat
    return out.reshape(planes.shape)


def dedup_tables(cub: torch.Tensor):
    """Per-pair spline tables [S*S, ...] -> (distinct tables [T, ...], int32 map [S*S] pair -> table).  Tables are
    merged only when bitwise identical, so the kernels read exactly the values they would read per pair; a model
    whose radial weights depend on the species pair keeps all S*S tables."""
    reps, idx = [], []
    for p in range(cub.shape[0]):
        for u, q in enumerate(reps):
            if torch.equal(cub[p], cub[q]):
                idx.append(u)
                break
        else:
            reps.append(p)
            idx.append(len(reps) - 1)
    tmap = torch.as_tensor(idx, dtype=torch.int32, device=cub.device)
    if len(reps) == cub.shape[0]:
        return cub, tmap
    return cub[reps].contiguous(), tmap


def tab2_pair_layout(cub: torch.Tensor) -> torch.Tensor:
    """Layer-2 cubic tables [T, M-1, nW * C, 4] (column w C + c, coefficients a, b, c, d) -> the paired layout the
    layer-2 kernels read: per interval [p][half][C] float4 with half 0 = (a_2p, a_2p+1, b_2p, b_2p+1) and
    half 1 = (c_2p, c_2p+1, d_2p, d_2p+1), so that paths 2p and 2p + 1 are evaluated with packed FP32x2 FMAs.
    Same size, same row offset per interval."""
    T, K, D, four = cub.shape
    nW = D // C
    assert four == 4 and D == nW * C and nW % 2 == 0
    x = cub.view(T, K, nW // 2, 2, C, 2, 2)                  # [t, k, p, path in pair, c, h, j]: coefficient 2 h + j
    return x.permute(0, 1, 2, 5, 4, 6, 3).contiguous().view(T, K, D, 4)


def fold_weights(model: Mdl.MACEModel, cols) -> dict:
    """All folded fp64 arrays (CPU numpy) for the species columns `cols` (model one-hot columns present)."""
    a = model.arch
    Zn = len(a.atomic_numbers)
    S = len(cols)
    P = {k: v.detach().double().numpy() for k, v in model.params().items()}
    cst = Mdl.silu_normalize2mom_cst()
    t1, t2 = Mdl.tp_tables()
    out = {"S": S, "cst": cst}
    for i in (0, 1):
        Ws = [P[f"interactions.{i}.conv_tp_weights.{k}"] for k in range(4)]
        out[f"A{i}"] = [Ws[0] / math.sqrt(Ws[0].shape[0])] + [cst * W / math.sqrt(W.shape[0]) for W in Ws[1:]]
        out[f"wd{i}"] = P[f"interactions.{i}.density_fn.weight"] / math.sqrt(a.num_bessel)
    emb = P["node_embedding.weight"][cols] / math.sqrt(Zn)                       # [S, C]
    X1 = emb @ P["interactions.0.linear_up.weight"][0] / math.sqrt(C)             # [S, C]
    out["X1"] = X1
    cs = np.zeros((S * S, t1["nW"] * C))
    for ss in range(S):
        for sr in range(S):
            cs[ss * S + sr] = np.tile(X1[ss], t1["nW"])
    out["col_scale1"] = cs
    Wl1 = P["interactions.0.linear.weight"]                                       # [4 mid entries, C, C]
    Wsk0 = P["interactions.0.skip_tp.weight"]                                     # [4, C, Z, C]
    M0 = np.zeros((S, 4, C, C))
    for s, z in enumerate(cols):
        for l in range(4):
            (w,) = t1["lin_groups"][l]
            M0[s, l] = (Wl1[w] / math.sqrt(C)) @ (Wsk0[l][:, z, :] / math.sqrt(C * Zn))
    out["M0"] = M0
    out["Wp1"] = P["products.0.linear.weight"] / math.sqrt(C)
    out["wr0"] = P["readouts.0.weight"] / math.sqrt(C)
    out["Wup2"] = P["interactions.1.linear_up.weight"] / math.sqrt(C)
    out["Wsk1"] = np.stack([P["interactions.1.skip_tp.weight"][0][:, z, :] for z in cols]) / math.sqrt(C * Zn)
    Wl2 = P["interactions.1.linear.weight"].copy()
    for l, ws in t2["lin_groups"].items():
        for w in ws:
            Wl2[w] = Wl2[w] / math.sqrt(len(ws) * C)
    out["Wlin2"] = Wl2
    out["Wp2"] = P["products.1.linear.weight"][0] / math.sqrt(C)
    out["W1r"] = P["readouts.1.linear_1.weight"] / math.sqrt(C)
    out["w2r"] = cst * P["readouts.1.linear_2.weight"] / math.sqrt(a.readout_mlp)
    out["e0"] = P["atomic_energies"][cols] + a.shift
    for blk, prefix, Ls in ((0, "products.0", (0, 1)), (1, "products.1", (0,))):
        ents = o3.sc_entries(Ls)
        coef = np.zeros((S, len(ents), C))
        for t, (L, M, nu, mono, row) in enumerate(ents):
            W = P[f"{prefix}.sc.{L}.{nu}"]                                        # [Z, K, C]
            coef[:, t, :] = np.einsum("k,skc->sc", row, W[cols])
        out[f"sc{blk}"] = coef
        out[f"sc{blk}_fp"] = o3.sc_fingerprint(ents)
    return out


L1_DENSITY_H = 64      # radial-MLP hidden width the density kernels are written for (2 species slots x 64 = C)


def sc_coef_layout(sc) -> np.ndarray:
    """Symmetric-contraction coefficients [S][NT][C] -> [S][ceil(NT / 4)][C][4] (zero padded): coefficient t of
    channel c at [t // 4][c][t % 4], so that the kernels load four consecutive coefficients per 16-byte load."""
    sc = np.asarray(sc, dtype=np.float64)
    S, nt, c = sc.shape
    nt4 = (nt + 3) // 4
    pad = np.zeros((S, nt4 * 4, c))
    pad[:, :nt] = sc
    return np.ascontiguousarray(pad.reshape(S, nt4, 4, c).transpose(0, 1, 3, 2))


def l1_density_supported(f: dict) -> bool:
    """The density-projection layer 1 keeps up to two species slots of 64 hidden features per receiver (K = C)."""
    return f["S"] <= 2 and f["A0"][3].shape[0] == L1_DENSITY_H


def fold_l1_density(f: dict) -> np.ndarray:
    """Composite layer-1 node matrices of the exact density projection, fp64 [S, 4, 2 H, C]:
    Kc[s_r, l][slot H + q, c'] = sum_c A3[q, l C + c] X1[slot, c] M0[s_r, l][c, c'] (rows of an absent slot are 0).

    Layer-1 sender features depend only on the sender species and the radial MLP's last layer is linear, so
    msg1[lm, c] = sum_e W1(r_e)[l, c] X1[s_e, c] Y_lm(e) = sum_{s, q} A3[q, l C + c] X1[s, c] B[s, q, lm] with the
    per-receiver densities B[s, q, lm] = sum_{e: s_e = s} h_q(r_e) Y_lm(e), h the MLP's last hidden layer
    (mace_onegpu/ace_layer1.py:2-16 derives it; :60-83 evaluates it).  x1 = msg1 M0[s_r] / (rho1 + 1) is then
    B Kc[s_r] / (rho1 + 1): the same GEMM shape as the direct path's M0 step (2 H = C = 128)."""
    A3 = f["A0"][3]                                           # [H, 4 C]
    H, S = A3.shape[0], f["S"]
    if 2 * H != C:
        raise ValueError(f"density layer 1 needs a {C // 2}-wide last hidden layer (got {H})")
    Kc = np.zeros((S, 4, 2 * H, C))
    for sr in range(S):
        for l in range(4):
            for s in range(S):
                Kc[sr, l, s * H:(s + 1) * H] = (A3[:, l * C:(l + 1) * C] * f["X1"][s][None, :]) @ f["M0"][sr, l]
    return Kc


class FoldedModel:
    """Device-resident folded model for one species subset (the ctypes mb_model_t points into its tensors)."""

    def __init__(self, model: Mdl.MACEModel, cols, spline_grid: int = 512, r_lo: float = 0.5, device="cuda",
                 use_tc: bool | None = None, l1_mode: str | None = None):
        L = N.lib()
        if use_tc is None:
            use_tc = os.environ.get("MACE_B200_TC", "1") != "0"
        if l1_mode is None:
            l1_mode = os.environ.get("MACE_B200_L1", "auto")
        if l1_mode not in ("auto", "direct", "density"):
            raise ValueError(f"l1_mode must be 'auto', 'direct' or 'density' (got {l1_mode!r})")
        self.cols = [int(c) for c in cols]
        self.device = torch.device(device)
        a = model.arch
        f = fold_weights(model, self.cols)
        for blk in (0, 1):
            n = N.c_i32()
            fp = N.c_u64()
            N.check(L.mace_b200_sc_layout(blk, N.byref(n), N.byref(fp)), "sc_layout")
            if n.value != f[f"sc{blk}"].shape[1] or fp.value != f[f"sc{blk}_fp"]:
                raise RuntimeError(f"symmetric contraction {blk}: library layout ({n.value}, {fp.value:#x}) does not match "
                                   f"the host folding ({f[f'sc{blk}'].shape[1]}, {f[f'sc{blk}_fp']:#x}); "
                                   "regenerate csrc/symcon_gen.cuh and rebuild")
        S = f["S"]
        self.S = S
        ok = l1_density_supported(f)
        if l1_mode == "density" and not ok:
            raise ValueError("the density-projection layer 1 needs at most 2 species and a 64-wide radial MLP")
        # layer 1 as per-receiver densities of the MLP's hidden features (exact; one 64-column table) or as direct
        # per-edge weights W1 * X1 (one 4 C-column table per sender species); auto = density where supported
        self.l1_density = ok if l1_mode == "auto" else l1_mode == "density"
        M0 = fold_l1_density(f) if self.l1_density else f["M0"]
        self.M = int(spline_grid)
        self.r_lo = float(r_lo)
        self.r_max = float(a.r_max)
        self.scale = float(a.scale)
        self.folded = f
        dev = self.device
        t = {}
        t["wd1"] = _f32(f["wd0"], dev)
        t["wd2"] = _f32(f["wd1"], dev)
        t["M0"] = _f32(M0, dev)
        t["M0T"] = _f32(np.ascontiguousarray(np.swapaxes(M0, -1, -2)), dev)
        t["Wp1"] = _f32(f["Wp1"], dev)
        t["Wp1T"] = _f32(np.ascontiguousarray(np.swapaxes(f["Wp1"], -1, -2)), dev)
        t["wr0"] = _f32(f["wr0"], dev)
        t["sc1"] = _f32(sc_coef_layout(f["sc0"]), dev)
        t["Wup2"] = _f32(f["Wup2"], dev)
        t["Wup2T"] = _f32(np.ascontiguousarray(np.swapaxes(f["Wup2"], -1, -2)), dev)
        t["Wsk1"] = _f32(f["Wsk1"], dev)
        t["Wsk1T"] = _f32(np.ascontiguousarray(np.swapaxes(f["Wsk1"], -1, -2)), dev)
        t["Wlin2"] = _f32(f["Wlin2"], dev)
        t["Wlin2T"] = _f32(np.ascontiguousarray(np.swapaxes(f["Wlin2"], -1, -2)), dev)
        t["sc2"] = _f32(sc_coef_layout(f["sc1"]), dev)
        t["Wp2"] = _f32(f["Wp2"], dev)
        t["Wp2T"] = _f32(np.ascontiguousarray(f["Wp2"].T), dev)
        t["W1r"] = _f32(f["W1r"], dev)
        t["w2r"] = _f32(f["w2r"], dev)
        t["e0"] = torch.as_tensor(f["e0"], dtype=torch.float64, device=dev).contiguous()
        for name, key, transpose in (("M0", "M0", False), ("Wp1", "Wp1", False), ("Wup2", "Wup2", False),
                                     ("Wsk1", "Wsk1", False), ("Wlin2", "Wlin2", False), ("Wp2", "Wp2", False)):
            W = M0 if key == "M0" else f[key]
            t[name + "_tc"] = torch.as_tensor(tc_planes(W), device=dev).contiguous()
            t[name + "T_tc"] = torch.as_tensor(tc_planes(np.swapaxes(W, -1, -2)), device=dev).contiguous()
        # spline tables built on the GPU in fp64: tab1 carries X1 of the sender species (direct layer 1) or is the
        # MLP's last hidden layer h(r) (density layer 1: last-layer matrix = identity, one table for all pairs)
        self.TV, self.TG = {}, {}
        for i, key, D, csk in ((0, "tab1", 4 * C, "col_scale1"), (1, "tab2", 10 * C, None)):
            A = [torch.as_tensor(x, dtype=torch.float64, device=dev).contiguous() for x in f[f"A{i}"]]
            cs = None if csk is None else torch.as_tensor(f[csk], dtype=torch.float64, device=dev).contiguous()
            npair = S * S
            if i == 0 and self.l1_density:
                D, cs, npair = L1_DENSITY_H, None, 1
                A[3] = torch.eye(L1_DENSITY_H, dtype=torch.float64, device=dev)
            TV = torch.empty(npair, self.M, D, dtype=torch.float32, device=dev)
            TG = torch.empty_like(TV)
            cub = torch.empty(npair, self.M - 1, D, 4, dtype=torch.float32, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            N.check(L.mace_b200_build_tables(N.ptr(A[0]), N.ptr(A[1]), N.ptr(A[2]), N.ptr(A[3]), A[0].shape[0],
                                             A[0].shape[1], D, N.ptr(cs), npair, self.M, self.r_lo, self.r_max,
                                             float(a.num_poly_cutoff), N.ptr(TV), N.ptr(TG), N.ptr(cub), st),
                    "build_tables")
            if npair == 1:
                t[key], t[key + "_map"] = cub, None
            else:
                t[key], t[key + "_map"] = dedup_tables(cub)
            if key == "tab2":
                t[key] = tab2_pair_layout(t[key])
            self.TV[i], self.TG[i] = TV, TG
            t[f"_A{i}"] = A
        self.t = t
        h = (self.r_max - self.r_lo) / (self.M - 1)
        self.struct = N.MBModel(C=C, S=S, M=self.M, r_lo=self.r_lo, inv_h=1.0 / h, r_max=self.r_max,
                                p_cut=float(a.num_poly_cutoff), scale=self.scale, use_tc=1 if use_tc else 0,
                                l1_density=1 if self.l1_density else 0,
                                **{k: N.ptr(v) for k, v in t.items() if not k.startswith("_")})
        self.use_tc = bool(use_tc)


class Plan:
    """Per-call preparation: receiver-sorted pairs, CSR, compact species, species-sorted chunk order.

    Pinned host pair arrays (pair_i / pair_j int32, rij fp64, contiguous) that look receiver-sorted stay on the host:
    the chunks' edge ranges come from a binary search of the pinned pair_i, and the evaluation streams every chunk's
    pairs to the device on a side stream, where mace_b200_csr_rows forms the chunk's rows and checks the
    sortedness the search assumed (host_src).  Anything else is copied here, sorted by receiver when needed
    (stable, like the reference's argsort, mliap_threepass.py:472-474) and its CSR formed on the device."""

    def __init__(self, eng: "ThreePassEngine", pair_i, pair_j, rij, elems, nl: int, nt: int, stream_host: bool = True):
        dev = eng.device
        self.nl, self.nt = int(nl), int(nt)
        self.P = int(pair_i.shape[0])
        self.perm = None
        self.host_src = None
        self._inputs = (pair_i, pair_j, rij, elems)
        C_ = eng.chunk
        nch = (self.nl + C_ - 1) // C_
        self.n_chunks = nch
        bounds = torch.clamp(torch.arange(nch + 1, dtype=torch.int64) * C_, max=self.nl)
        e_off = None
        if stream_host and self.P > 1 and nch > 0 and _pinned(pair_i, torch.int32) and \
                _pinned(pair_j, torch.int32) and _pinned(rij, torch.float64):
            hpi = pair_i.view(-1)
            e_off = torch.searchsorted(hpi, bounds.to(torch.int32)).numpy().astype(np.int64)
            if e_off[0] != 0 or e_off[-1] != self.P or bool((np.diff(e_off) < 0).any()):
                e_off = None                   # not receiver-sorted (or receivers outside [0, nl)): copy and sort
        if e_off is not None:
            self.host_src = (hpi, pair_j.view(-1), rij.view(-1, 3))
            self.pi = torch.empty(self.P, dtype=torch.int32, device=dev)
            self.pj = torch.empty(self.P, dtype=torch.int32, device=dev)
            self.rij = torch.empty(self.P, 3, dtype=torch.float64, device=dev)
            self.rowptr = torch.empty(self.nl + 1, dtype=torch.int32, device=dev)
            self.bounds = bounds.numpy()
        else:
            pi = torch.as_tensor(pair_i, device=dev).to(torch.int32)
            pj = torch.as_tensor(pair_j, device=dev).to(torch.int32)
            rr = torch.as_tensor(rij, device=dev).to(torch.float64)
            ordered = self.P <= 1 or bool((pi[1:] >= pi[:-1]).all())
            if not ordered:
                o = torch.argsort(pi, stable=True)
                pi, pj, rr = pi[o], pj[o], rr[o]
                self.perm = o.to(torch.int64).contiguous()
            self.pi, self.pj, self.rij = pi.contiguous(), pj.contiguous(), rr.reshape(-1, 3).contiguous()
            self.rowptr = torch.searchsorted(pi, torch.arange(self.nl + 1, device=dev, dtype=torch.int32)).to(torch.int32)
            e_off = self.rowptr[bounds.to(dev)].to(torch.int64).cpu().numpy()
            if self.P and (e_off[0] != 0 or e_off[-1] != self.P):
                raise RuntimeError(f"Plan: pair_i holds receivers outside [0, nlocal = {self.nl})")
        self.e_off = e_off                                              # edge range of every chunk (host)
        el = torch.as_tensor(elems, device=dev).to(torch.int64)
        zn = eng.col2s.numel()
        spec = torch.where((el >= 0) & (el < zn), eng.col2s[el.clamp(0, zn - 1)], -1)
        self.spec = spec.to(torch.int32).contiguous()
        S = eng.fm.S
        cid = torch.arange(self.nl, device=dev) // C_
        key = cid * S + self.spec[:self.nl].long()
        og = torch.argsort(key, stable=True)
        self.order = (og - cid[og] * C_).to(torch.int32).contiguous()
        # one device -> host read: species counts per chunk plus the number of atoms without tables
        cnt = torch.cat([torch.bincount(key, minlength=max(nch * S, 1)), (spec < 0).sum().view(1)]).cpu().numpy()
        if cnt[-1]:
            raise RuntimeError("Plan: an atom's species has no tables in this engine (rebuild it with that species)")
        cnt = cnt[:-1].reshape(max(nch, 1), S)
        off = np.zeros((max(nch, 1), S + 1), dtype=np.int32)
        off[:, 1:] = np.cumsum(cnt, 1)
        self.spec_off = np.ascontiguousarray(off.reshape(-1))

    def sorted_copy(self, eng: "ThreePassEngine") -> "Plan":
        """The same inputs copied to the device and sorted there (after MB_ST_UNSORTED from a streamed plan)."""
        return Plan(eng, *self._inputs, self.nl, self.nt, stream_host=False)


def pipeline_steps(nch: int, chunk: int, nl: int, largest_sender, lookahead: int = 2):
    """Order of the pipelined pass A / pass B schedule of a streamed pair list (ThreePassEngine._run_pipelined).
    Pass-B chunk c reads the X2 rows of its senders only, so it can run once pass A (and the X2 GEMM of its rows)
    has covered the chunks up to need(c) = max(c, largest sender of c // chunk); a chunk with a ghost sender
    (index >= nl) needs the H1 exchange, which follows the last pass-A chunk.  largest_sender(c) is -1 for a chunk
    without pairs and may block until the chunk has arrived: it is called for chunk k - lookahead + 1 right after
    pass-A chunk k is issued (the host stays `lookahead` chunks ahead of the arrivals), then for the rest.
    Yields ("A", k), ("early_B", c) for a pass-B chunk issued before the last pass-A chunk, ("exchange", None)
    once after the last pass-A chunk, and ("B", c) for the others.  With spatially sorted atoms (LAMMPS sorts them
    into bins) need(c) is c + 2 or c + 3 for almost every chunk, so the pair list's host-to-device transfer hides
    under pass B instead of under pass A alone."""
    pend = []                 # heap of (need, chunk) for chunks whose sender range is known
    known = 0

    def learn(upto):
        nonlocal known
        while known < upto:
            hi = int(largest_sender(known))
            need = known if hi < 0 else nch if hi >= nl else max(known, hi // chunk)
            heapq.heappush(pend, (need, known))
            known += 1

    for k in range(nch):
        yield "A", k
        learn(max(0, k + 1 - lookahead))
        while pend and pend[0][0] <= k:
            yield ("early_B" if k < nch - 1 else "B"), heapq.heappop(pend)[1]
    yield "exchange", None
    learn(nch)
    while pend:
        yield "B", heapq.heappop(pend)[1]


def _pinned(t, dtype) -> bool:
    return isinstance(t, torch.Tensor) and not t.is_cuda and t.is_pinned() and t.dtype == dtype and t.is_contiguous()


class ThreePassEngine:
    """The three-pass evaluation on one GPU for a fixed model and species set."""

    def __init__(self, model: Mdl.MACEModel, cols, chunk: int = 16384, spline_grid: int = 512, device="cuda",
                 use_tc: bool | None = None, x1_cache: bool | None = None, l1_mode: str | None = None):
        self.device = torch.device(device)
        self.model = model
        self.chunk = int(chunk)
        # cache pass A's layer-1 intermediates for pass C when they fit comfortably (8 KB per local atom); None = auto
        env = os.environ.get("MACE_B200_X1_CACHE")
        self.x1_cache = x1_cache if x1_cache is not None else (None if env is None else env != "0")
        self.graphs = os.environ.get("MACE_B200_GRAPHS", "0") == "1"
        # streamed single-GPU pair lists: run every pass-B chunk as soon as pass A has covered its senders
        self.pipeline = os.environ.get("MACE_B200_PIPELINE", "1") != "0"
        self._dep_host = None
        self.last_schedule = None         # "serial", "overlap", "pipelined" or "graph": how the last call ran
        self.early_b_chunks = 0           # pipelined: pass-B chunks issued before pass A's last chunk
        self._graph = None
        self.captures = 0
        self.fm = FoldedModel(model, cols, spline_grid=spline_grid, device=self.device, use_tc=use_tc, l1_mode=l1_mode)
        Zn = len(model.arch.atomic_numbers)
        col2s = torch.full((Zn,), -1, dtype=torch.int64)
        col2s[torch.as_tensor(self.fm.cols)] = torch.arange(len(self.fm.cols))
        self.col2s = col2s.to(self.device)
        self._buf = {}
        self._cap = {}
        self._io = None                   # side stream of the host <-> device copies
        self.pass_timing = False          # record CUDA events between the passes (pass_times())
        self._marks = None
        self._marks_valid = False
        self._h2d_marks = None
        self._ev_cache = {}
        self.host_pf_written = False

    # ------------------------------------------------------------------------------------------------ buffers
    def _get(self, name, shape, dtype):
        n = int(np.prod(shape))
        b = self._buf.get(name)
        if b is None or b.numel() < n or b.dtype != dtype:
            b = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self._buf[name] = b
        return b[:n].view(*shape)

    def plan(self, pair_i, pair_j, rij, elems, nl, nt) -> Plan:
        return Plan(self, pair_i, pair_j, rij, elems, nl, nt)

    def eval_struct(self, plan: Plan):
        nl, nt, P, ch = plan.nl, plan.nt, plan.P, self.chunk
        f32, f64 = torch.float32, torch.float64
        b = dict(H1=self._get("H1", (nt, 4, C), f32), X2=self._get("X2", (nt, 4, C), f32),
                 G1=self._get("G1", (nt, 4, C), f32), GX2=self._get("GX2", (nt, 4, C), f32),
                 PF=self._get("PF", (P, 3), f32), eat=self._get("eat", (max(nl, 1),), f64),
                 s_msg=self._get("s_msg", (ch, 40, C), f32), s_x=self._get("s_x", (ch, 16, C), f32),
                 s_gx=self._get("s_gx", (ch, 16, C), f32), s_a=self._get("s_a", (ch, 4, C), f32),
                 s_ga=self._get("s_ga", (ch, 4, C), f32), s_h=self._get("s_h", (ch, C), f32),
                 s_gh=self._get("s_gh", (ch, C), f32), s_sc=self._get("s_sc", (ch, C), f32),
                 s_rho=self._get("s_rho", (ch,), f32), s_grho=self._get("s_grho", (ch,), f32),
                 status=self._get("status", (1,), torch.int32))
        if self._use_x1_cache(nl):
            b["x1_cache"] = self._get("x1_cache", (max(nl, 1), 16, C), f32)
            b["rho1_cache"] = self._get("rho1_cache", (max(nl, 1),), f32)
        ev = N.MBEval(nl=nl, nt=nt, P=P, pair_i=N.ptr(plan.pi), pair_j=N.ptr(plan.pj), rij=N.ptr(plan.rij),
                      rowptr=N.ptr(plan.rowptr), spec=N.ptr(plan.spec), chunk=ch, order=N.ptr(plan.order),
                      spec_off=plan.spec_off.ctypes.data, **{k: N.ptr(v) for k, v in b.items()})
        return ev, b

    def _use_x1_cache(self, nl: int) -> bool:
        if self.x1_cache is not None:
            return bool(self.x1_cache)
        have = self._buf.get("x1_cache")
        if have is not None and have.numel() >= nl * 16 * C:
            return True
        free, _total = torch.cuda.mem_get_info(self.device)
        return nl * 16 * C * 4 < 0.25 * free

    def _check_status(self, b, what):
        s = int(b["status"].item())
        if s:
            names = [n for bit, n in ((1, "sender index out of range"), (2, "species out of range"),
                                      (4, "bad CSR row pointer"), (8, "non-finite or zero edge vector"),
                                      (16, "pair_i does not match its CSR row"),
                                      (32, "tensor-core GEMM barrier wait expired"),
                                      (64, "pair_i not sorted by receiver")) if s & bit]
            raise RuntimeError(f"mace_b200 {what}: input error reported by the kernels: {', '.join(names)}")

    # ------------------------------------------------------------------------------------------------ evaluation
    def _run(self, plan, ev, b, forward_exchange=None, reverse_exchange=None, zero_status=True):
        """The device work of one evaluation on the current stream (capturable when there is no exchange)."""
        L = N.lib()
        m = N.byref(self.fm.struct)
        evp = N.byref(ev)
        st = torch.cuda.current_stream(self.device).cuda_stream
        if zero_status:
            b["status"].zero_()
        b["eat"].zero_()
        PFd = self._get("PFd", (plan.P, 3), torch.float64)
        fbits = self._get("fmax", (1,), torch.int32)
        fbits.zero_()
        if ev.done_ev:                                   # pass C hands out every finished chunk's pair forces
            ev.pf_out, ev.fmax_bits = N.ptr(PFd), N.ptr(fbits)
        marks = self._pass_marks() if self.pass_timing and not torch.cuda.is_current_stream_capturing() else None
        self._marks_valid = marks is not None
        mark = (lambda k: marks[k].record()) if marks else (lambda k: None)
        mark(0)
        N.check(L.mace_b200_pass_a(m, evp, st), "pass_a")
        mark(1)
        if forward_exchange is not None and plan.nt > plan.nl:
            forward_exchange(b["H1"].view(plan.nt, 4 * C))
        mark(2)
        N.check(L.mace_b200_x2_all(m, evp, st), "x2_all")
        N.check(L.mace_b200_pass_b(m, evp, st), "pass_b")
        mark(3)
        if reverse_exchange is not None and plan.nt > plan.nl:
            reverse_exchange(b["G1"].view(plan.nt, 4 * C))
        mark(4)
        N.check(L.mace_b200_pass_c(m, evp, st), "pass_c")
        mark(5)
        N.check(L.mace_b200_finalize(m, evp, N.ptr(plan.perm), N.ptr(PFd), N.ptr(fbits), st), "finalize")
        mark(6)
        return PFd, fbits

    def _run_overlap(self, plan, ev, b, halo):
        """The evaluation with both halo exchanges overlapped with interior chunks.  Chunk k holds local atoms
        [k chunk, (k + 1) chunk); chunks [0, kI) hold interior atoms only (no ghost senders, and no rank receives
        their rows), the rest hold the boundary atoms.  Main stream / side stream:
            pass A boundary chunks                  -> side: H1 forward exchange
            pass A interior chunks, X2 of local rows, pass B interior chunks
            (wait forward) X2 of ghost rows, pass B boundary chunks, fold of the ghost rows of G1
                                                    -> side: G1 reverse exchange (communication)
            fold of the local rows of G1, pass C interior chunks
            (wait reverse) received ghost rows added onto their owners, pass C boundary chunks, finalize.
        Every rank issues the same exchanges in the same order."""
        L = N.lib()
        m = N.byref(self.fm.struct)
        evp = N.byref(ev)
        cur = torch.cuda.current_stream(self.device)
        st = cur.cuda_stream
        if getattr(self, "_halo_stream", None) is None:
            self._halo_stream = torch.cuda.Stream(self.device)
        side = self._halo_stream
        nl, nt, nch = plan.nl, plan.nt, plan.n_chunks
        kI = min(int(halo.n_interior) // self.chunk, nch)
        self._marks_valid = False
        b["eat"].zero_()
        PFd = self._get("PFd", (plan.P, 3), torch.float64)
        fbits = self._get("fmax", (1,), torch.int32)
        fbits.zero_()
        H1 = b["H1"].view(nt, 4 * C)
        G1 = b["G1"].view(nt, 4 * C)
        e_a, e_fwd, e_b, e_rev = (torch.cuda.Event() for _ in range(4))
        N.check(L.mace_b200_pass_a_chunks(m, evp, kI, nch, st), "pass_a")
        e_a.record(cur)
        with torch.cuda.stream(side):
            side.wait_event(e_a)
            halo.forward(H1)
            e_fwd.record(side)
        N.check(L.mace_b200_pass_a_chunks(m, evp, 0, kI, st), "pass_a")
        N.check(L.mace_b200_x2_rows(m, evp, 0, nl, st), "x2_rows")
        b["PF"].zero_()
        N.check(L.mace_b200_pass_b_chunks(m, evp, 0, kI, st), "pass_b")
        cur.wait_event(e_fwd)
        N.check(L.mace_b200_x2_rows(m, evp, nl, nt, st), "x2_rows")
        N.check(L.mace_b200_pass_b_chunks(m, evp, kI, nch, st), "pass_b")
        N.check(L.mace_b200_fold_g1(m, evp, nl, nt, st), "fold_g1")
        e_b.record(cur)
        with torch.cuda.stream(side):
            side.wait_event(e_b)
            halo.reverse_comm(G1)
            e_rev.record(side)
        N.check(L.mace_b200_fold_g1(m, evp, 0, nl, st), "fold_g1")
        N.check(L.mace_b200_pass_c_chunks(m, evp, 0, kI, st), "pass_c")
        cur.wait_event(e_rev)
        halo.reverse_unpack(G1)
        N.check(L.mace_b200_pass_c_chunks(m, evp, kI, nch, st), "pass_c")
        N.check(L.mace_b200_finalize(m, evp, N.ptr(plan.perm), N.ptr(PFd), N.ptr(fbits), st), "finalize")
        return PFd, fbits

    _LOOKAHEAD = 2      # pipelined schedule: pass A chunk k is issued once chunk k - 2's sender range is known

    def _run_pipelined(self, plan, ev, b, dep_host, ready, forward_exchange=None, reverse_exchange=None):
        """Evaluation of a streamed pair list with pass B interleaved into pass A (the order: pipeline_steps).  The
        side stream reports each chunk's sender range (mace_b200_sender_range) together with its arrival; the host
        reads a chunk's largest sender once the chunk has arrived.  Pass C follows all of pass B.  Timing marks: t_A
        covers pass A with the pass-B chunks interleaved in it, t_B the remaining pass-B chunks and the G1 fold."""
        L = N.lib()
        m = N.byref(self.fm.struct)
        evp = N.byref(ev)
        st = torch.cuda.current_stream(self.device).cuda_stream
        nl, nch, C_ = plan.nl, plan.n_chunks, self.chunk
        b["eat"].zero_()
        b["PF"].zero_()
        PFd = self._get("PFd", (plan.P, 3), torch.float64)
        fbits = self._get("fmax", (1,), torch.int32)
        fbits.zero_()
        if ev.done_ev:
            ev.pf_out, ev.fmax_bits = N.ptr(PFd), N.ptr(fbits)
        marks = self._pass_marks() if self.pass_timing else None
        self._marks_valid = marks is not None
        mark = (lambda k: marks[k].record()) if marks else (lambda k: None)

        def largest_sender(c):
            ready[c].synchronize()
            return int(dep_host[c, 1])

        mark(0)
        self.early_b_chunks = 0
        for kind, k in pipeline_steps(nch, C_, nl, largest_sender, self._LOOKAHEAD):
            if kind == "A":
                N.check(L.mace_b200_pass_a_chunks(m, evp, k, k + 1, st), "pass_a")
                N.check(L.mace_b200_x2_rows(m, evp, k * C_, min((k + 1) * C_, nl), st), "x2_rows")
            elif kind == "early_B" or kind == "B":
                N.check(L.mace_b200_pass_b_chunks(m, evp, k, k + 1, st), "pass_b")
                self.early_b_chunks += kind == "early_B"
            else:                                   # "exchange": after the last pass-A chunk
                mark(1)
                if plan.nt > nl:
                    if forward_exchange is not None:
                        forward_exchange(b["H1"].view(plan.nt, 4 * C))
                    N.check(L.mace_b200_x2_rows(m, evp, nl, plan.nt, st), "x2_rows")
                mark(2)
        N.check(L.mace_b200_fold_g1(m, evp, 0, plan.nt, st), "fold_g1")
        mark(3)
        if reverse_exchange is not None and plan.nt > nl:
            reverse_exchange(b["G1"].view(plan.nt, 4 * C))
        mark(4)
        N.check(L.mace_b200_pass_c(m, evp, st), "pass_c")
        mark(5)
        N.check(L.mace_b200_finalize(m, evp, N.ptr(plan.perm), N.ptr(PFd), N.ptr(fbits), st), "finalize")
        mark(6)
        return PFd, fbits

    _PASSES = ("A", "xchg_fwd", "B", "xchg_rev", "C", "finalize")

    def _pass_marks(self):
        if self._marks is None:
            self._marks = [torch.cuda.Event(enable_timing=True) for _ in range(len(self._PASSES) + 1)]
        return self._marks

    def pass_times(self) -> dict:
        """Seconds of each pass of the last eager evaluation (CUDA events; needs pass_timing = True before it ran,
        the per-pass timers of the reference's log, mliap_threepass.py:488-587).  Synchronises."""
        if not self._marks or not self._marks_valid:
            return {}
        self._marks[-1].synchronize()
        out = {f"t_{name}": self._marks[k].elapsed_time(self._marks[k + 1]) * 1e-3
               for k, name in enumerate(self._PASSES)}
        if self._h2d_marks is not None:           # streamed pair list: its side-stream copies (all chunks)
            self._h2d_marks[1].synchronize()
            out["t_h2d_pairs"] = self._h2d_marks[0].elapsed_time(self._h2d_marks[1]) * 1e-3
            out["t_h2d_pairs_after_A_start"] = self._marks[0].elapsed_time(self._h2d_marks[1]) * 1e-3
            self._h2d_marks = None
        return out

    def _events(self, key, n):
        evs = self._ev_cache.get(key)
        if evs is None or len(evs) < n:
            evs = [torch.cuda.Event() for _ in range(n)]
            cur = torch.cuda.current_stream(self.device)
            for e in evs:                               # materialise the handles the library records / waits on
                e.record(cur)
            self._ev_cache[key] = evs
        return evs[:n]

    def evaluate(self, plan: Plan, forward_exchange=None, reverse_exchange=None, check: bool = True,
                 graph: bool | None = None, host_pf=None, halo=None):
        """(eatoms fp64 [nl], pair forces dE/drij fp64 [P, 3] in the caller's pair order) on the device.
        forward_exchange(H1 [nt, 512]) fills ghost rows from their owners; reverse_exchange(G1 [nt, 512]) adds
        ghost rows onto their owners (both in place; None when nt == nl).  graph=True (or engine.graphs) replays
        the whole evaluation as one captured CUDA graph when there is no exchange to run between the passes.

        halo (instead of the two callbacks): an exchange object with forward(H), reverse_comm(G), reverse_unpack(G)
        and n_interior, whose local atoms [0, n_interior) have no ghost neighbours (domain.HaloExchange).  The
        exchanges then run on a side stream, overlapped with interior work (_run_overlap).

        Host I/O overlap: a plan whose senders / vectors are in pinned host memory (Plan.host_src) gets them copied
        chunk by chunk on a side stream, pass A waiting per chunk; with host_pf (pinned fp64 [P, 3]) and
        receiver-sorted input, every chunk's final pair forces are copied into host_pf as soon as pass C has
        finished the chunk (self.host_pf_written tells whether that happened; the returned device array is then
        complete as well)."""
        self.host_pf_written = False
        deferred = plan.host_src is not None
        use_graph = self.graphs if graph is None else graph
        if use_graph and forward_exchange is None and reverse_exchange is None and not deferred:
            self.last_schedule = "graph"
            b, PFd, fbits = self._evaluate_graph(plan)
        else:
            ev, b = self.eval_struct(plan)
            cur = torch.cuda.current_stream(self.device)
            e_off, nch = plan.e_off, plan.n_chunks
            keep = []
            b["status"].zero_()                           # before the side stream's CSR checks can set bits
            if deferred or host_pf is not None:
                if self._io is None:
                    # high priority: its small CSR / sender-range kernels must not queue behind the pass kernels
                    self._io = torch.cuda.Stream(self.device, priority=-1)
                io = self._io
                io.wait_stream(cur)
            pipe = deferred and self.pipeline and not (halo is not None and plan.nt > plan.nl) and nch > 1
            if deferred:
                ops = N.ops()
                h_pi, h_pj, h_rij = plan.host_src
                waits = self._events("wait", nch)
                if pipe:
                    dep_dev = self._get("sender_range", (nch, 2), torch.int32)
                    if self._dep_host is None or self._dep_host.shape[0] < nch:
                        self._dep_host = torch.empty(nch, 2, dtype=torch.int32, pin_memory=True)
                    dep_host = self._dep_host
                with torch.cuda.stream(io):
                    if self.pass_timing:
                        self._h2d_marks = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
                        self._h2d_marks[0].record(io)
                    for k in range(nch):
                        e0, e1 = int(e_off[k]), int(e_off[k + 1])
                        plan.pi[e0:e1].copy_(h_pi[e0:e1], non_blocking=True)
                        plan.pj[e0:e1].copy_(h_pj[e0:e1], non_blocking=True)
                        plan.rij[e0:e1].copy_(h_rij[e0:e1], non_blocking=True)
                        ops.csr_rows(plan.pi, e0, e1, int(plan.bounds[k]), int(plan.bounds[k + 1]), plan.rowptr,
                                     b["status"])
                        if pipe:
                            N.check(N.lib().mace_b200_sender_range(N.ptr(plan.pj), e0, e1, N.ptr(dep_dev[k]),
                                                                   io.cuda_stream), "sender_range")
                            dep_host[k].copy_(dep_dev[k], non_blocking=True)
                        waits[k].record(io)
                    if self.pass_timing:
                        self._h2d_marks[1].record(io)
                for t in (plan.pi, plan.pj, plan.rij, plan.rowptr, b["status"]) + ((dep_dev,) if pipe else ()):
                    t.record_stream(io)
                arr = (N.ctypes.c_void_p * nch)(*[e.cuda_event for e in waits])
                keep.append(arr)
                ev.wait_ev = N.ctypes.addressof(arr)
            out_host = host_pf is not None and plan.perm is None and nch > 0
            if out_host:
                done = self._events("done", nch)
                arr2 = (N.ctypes.c_void_p * nch)(*[e.cuda_event for e in done])
                keep.append(arr2)
                ev.done_ev = N.ctypes.addressof(arr2)
            self.last_schedule = "overlap" if halo is not None and plan.nt > plan.nl else \
                "pipelined" if pipe else "serial"
            if self.last_schedule == "overlap":
                PFd, fbits = self._run_overlap(plan, ev, b, halo)
            elif pipe:
                PFd, fbits = self._run_pipelined(plan, ev, b, dep_host, waits, forward_exchange, reverse_exchange)
            else:
                PFd, fbits = self._run(plan, ev, b, forward_exchange, reverse_exchange, zero_status=False)
            if out_host:
                with torch.cuda.stream(io):
                    for k in range(nch):
                        e0, e1 = int(e_off[k]), int(e_off[k + 1])
                        io.wait_event(done[k])
                        host_pf[e0:e1].copy_(PFd[e0:e1], non_blocking=True)
                PFd.record_stream(io)
                self.host_pf_written = True
            if deferred or out_host:
                cur.wait_stream(io)
        self._last = b
        if deferred and int(b["status"].item()) & N.ST_UNSORTED:
            # the streamed pair list was not receiver-sorted after all: evaluate again from a sorted device copy
            return self.evaluate(plan.sorted_copy(self), forward_exchange, reverse_exchange, check, graph, host_pf)
        if check:
            self._check_status(b, "evaluation")
        self.fmax = float(fbits.view(torch.float32).item()) if check else None
        return b["eat"][:plan.nl], PFd

    # ------------------------------------------------------------------------------------------------ CUDA graph
    _STAGED = ("pi", "pj", "rij", "rowptr", "spec", "order")

    def _evaluate_graph(self, plan: Plan):
        """Capture (once per shape / species layout) and replay the evaluation.  The plan's device arrays are copied
        into persistent staging buffers whose addresses the graph holds; the species segment table (host) is part of
        the capture key because the chunk loops bake it into the launch parameters."""
        key = (plan.P, plan.nl, plan.nt, plan.perm is not None, plan.spec_off.tobytes())
        g = self._graph
        if g is None or g["key"] != key:
            self._graph = None
            staged = Plan.__new__(Plan)
            staged.P, staged.nl, staged.nt, staged.n_chunks = plan.P, plan.nl, plan.nt, plan.n_chunks
            staged.spec_off = plan.spec_off.copy()
            for name in self._STAGED:
                setattr(staged, name, getattr(plan, name).clone())
            staged.perm = None if plan.perm is None else plan.perm.clone()
            ev, b = self.eval_struct(staged)
            self._run(staged, ev, b)                            # eager warm-up (one-time kernel attributes)
            torch.cuda.synchronize(self.device)
            gr = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                with torch.cuda.graph(gr, stream=side):
                    PFd, fbits = self._run(staged, ev, b)
            torch.cuda.current_stream(self.device).wait_stream(side)
            g = self._graph = dict(key=key, graph=gr, staged=staged, ev=ev, b=b, PFd=PFd, fbits=fbits)
            self.captures += 1
        else:
            st = g["staged"]
            for name in self._STAGED:
                getattr(st, name).copy_(getattr(plan, name), non_blocking=True)
            if plan.perm is not None:
                st.perm.copy_(plan.perm, non_blocking=True)
        g["graph"].replay()
        self._marks_valid = False
        return g["b"], g["PFd"], g["fbits"]

    def owner_exchange(self, owner, nl: int):
        """Exchange callbacks for ghosts given by an owner map (owner[j] = local owner of atom j for j >= nl): the
        single-process stand-in of LAMMPS' forward / reverse comm (mliap_threepass.py:40-55, 522, 556)."""
        L = N.lib()
        ghost = torch.as_tensor(owner, device=self.device)[nl:].to(torch.int32).contiguous()

        def fwd(H):
            st = torch.cuda.current_stream(self.device).cuda_stream
            N.check(L.mace_b200_pack_rows(N.ptr(H), N.ptr(ghost), ghost.numel(), H.shape[1], N.ptr(H[nl:]), st),
                    "pack_rows")

        def rev(G):
            st = torch.cuda.current_stream(self.device).cuda_stream
            N.check(L.mace_b200_unpack_add_rows(N.ptr(G[nl:]), N.ptr(ghost), ghost.numel(), G.shape[1], N.ptr(G), st),
                    "unpack_add_rows")

        return fwd, rev
