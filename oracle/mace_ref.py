"""TEST INFRASTRUCTURE (oracle): CPU fp64 restatement of the reference's exact three-pass MACE force evaluation.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may import this module.  It is the checker of
the CUDA path (and the timed CPU baseline), never part of it.

What it restates (reference citations are paths inside ShiQiaoL/mace-million):
* the per-chunk layer math of ``mace_onegpu/receiver_chunk_mace.py:237-256`` (layer1 / layer2_energy) in the
  receiver-only order of ``mace_onegpu/fast_layers.py:168-222`` (density normalisation, L1 skip on the message,
  L2 skip as residual), with the mace-torch 0.3.15 blocks it calls restated from their published definitions:
  Bessel x polynomial cutoff, e3nn FullyConnectedNet radial MLP (normalize2mom SiLU, no biases,
  ``mace_onegpu/fused_radial.py:4-9``), channelwise 'uvu' tensor product, e3nn Linear (1/sqrt(fan_in)),
  FullyConnectedTensorProduct skip with one-hot species, symmetric contraction (U tensors x per-species weights),
  linear / non-linear readouts, scale-shift and E0;
* the three-pass driver of ``mace_onegpu/receiver_chunk_mace.py:278-386`` and ``mace_onegpu/mliap_threepass.py:444-605``
  (pass A -> H1 forward exchange -> pass B with dE/dvec, dE/dh1 -> G1 reverse exchange -> pass C with
  loss = E1 + G1 . h1), on the ML-IAP data model (receivers local, senders local or ghost, pair forces dE/drij);
* the tabulated radial weights of ``mace_onegpu/conv_spline.py:230-249`` / ``mace_onegpu/spline_radial.py:237-272``
  (fp64 samples on M knots over [0.5, r_max], dW/dr by central differences with eps = 1e-5 (r_hi - r_lo), cubic Hermite
  evaluation with x clamped to [0, M - 1 - 1e-4] as in ``mace_onegpu/spline_w.py:18-27``, the derivative taken at
  the clamped point as the reference's backward kernel does, ``spline_w.py:53-75``).

Pinning: the reference's own driver code (ThreePassMLIAP.compute_forces with FastLayers, ReceiverChunkMACE with
FastLayers and with ace_layer1's density-projection layer 1, conv_spline.build_tables, spline_radial._hermite_eval,
_exchange) was run on the CPU with this module's blocks behind
mace-torch's module interface (tests/golden/make_reference_pins.py); this restatement reproduces its outputs to
fp64 round-off (tests/test_reference_pins.py), which pins the three-pass driver, the layer order, the ML-IAP
semantics and the tables against the reference itself.  The block math (mace-torch / e3nn, not installed) stays
unpinned; the invariants the reference's own tests check (three-pass == full graph, chunk invariance, periodic
replica, fp32 vs fp64) plus rotation / inversion invariance and finite differences pin it (tests/test_oracle.py).
"""
from __future__ import annotations

import math

import torch

from . import o3_ref

C_TARGET = [(0, 1), (1, -1), (2, 1), (3, -1)]
C_HIDDEN = [(0, 1), (1, -1)]


def normalize2mom_silu() -> float:
    from scipy import integrate

    f = lambda z: (z / (1.0 + math.exp(-z))) ** 2 * math.exp(-0.5 * z * z) / math.sqrt(2.0 * math.pi)
    m2 = sum(integrate.quad(f, lo, hi, epsabs=0.0, epsrel=1e-13, limit=400)[0] for lo, hi in ((-40.0, 0.0), (0.0, 40.0)))
    return 1.0 / math.sqrt(m2)


def sh_torch(vec: torch.Tensor):
    """[E, 16] component-normalised real SH of the direction of vec (differentiable)."""
    r = torch.linalg.vector_norm(vec, dim=-1, keepdim=True)
    u = vec / r
    x, y, z = u[:, 0], u[:, 1], u[:, 2]
    r15, r5 = math.sqrt(15.0), math.sqrt(5.0)
    a0 = r15 * x * z
    a4 = 0.5 * r15 * (z * z - x * x)
    q = x * x + z * z
    cols = [torch.ones_like(x), math.sqrt(3.0) * x, math.sqrt(3.0) * y, math.sqrt(3.0) * z,
            a0, r15 * x * y, r5 * (y * y - 0.5 * q), r15 * y * z, a4,
            math.sqrt(42.0) / 6.0 * (a0 * z + a4 * x), math.sqrt(7.0) * a0 * y,
            math.sqrt(168.0) / 8.0 * (4.0 * y * y - q) * x, 0.5 * math.sqrt(7.0) * y * (2.0 * y * y - 3.0 * q),
            math.sqrt(168.0) / 8.0 * z * (4.0 * y * y - q), math.sqrt(7.0) * a4 * y,
            math.sqrt(42.0) / 6.0 * (a4 * z - a0 * x)]
    return torch.stack(cols, -1)


def _lsl(l):
    return slice(l * l, (l + 1) * (l + 1))


class MaceRef:
    """fp64 evaluator of the two-layer MACE given its parameters (dotted-name dict) and architecture dict."""

    def __init__(self, params: dict, arch: dict, spline_knots: int = 0, species_cols=None, r_lo: float = 0.5):
        self.P = {k: torch.as_tensor(v, dtype=torch.float64) for k, v in params.items()}
        self.a = dict(arch)
        self.C = int(arch["channels"])
        self.Z = len(arch["atomic_numbers"])
        self.rmax = float(arch["r_max"])
        self.nb = int(arch["num_bessel"])
        self.pcut = float(arch["num_poly_cutoff"])
        self.scale = float(arch["scale"])
        self.shift = float(arch["shift"])
        self.cst = normalize2mom_silu()
        self.inst = [o3_ref.tp_instructions([(0, 1)], C_TARGET), o3_ref.tp_instructions(C_HIDDEN, C_TARGET)]
        self.w3 = {}
        for insts, nirr in ((self.inst[0], [(0, 1)]), (self.inst[1], C_HIDDEN)):
            for (lo, i1, i2) in insts:
                l1 = nirr[i1][0]
                self.w3[(l1, i2, lo)] = torch.as_tensor(o3_ref.w3j(l1, i2, lo) * math.sqrt(2 * lo + 1))
        self.U = {(L, nu): torch.as_tensor(o3_ref.U(nu, L)) for L in (0, 1) for nu in (1, 2, 3)}
        self.knots = int(spline_knots)
        self.r_lo = float(r_lo)
        self.tables = None
        if self.knots:
            self.tables = [self._build_table(i) for i in (0, 1)]

    # ------------------------------------------------------------------------------------------ radial parts
    def bessel_cut(self, r: torch.Tensor) -> torch.Tensor:
        """edge_feats = Bessel(r) * f_cut(r), [E, nb]."""
        n = torch.arange(1, self.nb + 1, dtype=torch.float64)
        b = math.sqrt(2.0 / self.rmax) * torch.sin(n * math.pi / self.rmax * r) / r
        p = self.pcut
        x = r / self.rmax
        env = (1.0 - (p + 1.0) * (p + 2.0) / 2.0 * x ** p + p * (p + 2.0) * x ** (p + 1.0)
               - p * (p + 1.0) / 2.0 * x ** (p + 2.0))
        return b * (env * (r < self.rmax))

    def radial_mlp(self, i: int, feats: torch.Tensor) -> torch.Tensor:
        h = feats
        k = 0
        while f"interactions.{i}.conv_tp_weights.{k + 1}" in self.P:
            W = self.P[f"interactions.{i}.conv_tp_weights.{k}"]
            h = self.cst * torch.nn.functional.silu(h @ W / math.sqrt(W.shape[0]))
            k += 1
        W = self.P[f"interactions.{i}.conv_tp_weights.{k}"]
        return h @ W / math.sqrt(W.shape[0])

    def density(self, i: int, feats: torch.Tensor) -> torch.Tensor:
        w = self.P[f"interactions.{i}.density_fn.weight"]
        d = feats @ w.unsqueeze(-1) / math.sqrt(w.shape[0])
        return torch.tanh(d * d)

    def _build_table(self, i: int):
        M = self.knots
        h = (self.rmax - self.r_lo) / (M - 1)
        eps = 1e-5 * (self.rmax - self.r_lo)
        r = torch.linspace(self.r_lo, self.rmax, M, dtype=torch.float64).unsqueeze(-1)
        with torch.no_grad():
            v0 = self.radial_mlp(i, self.bessel_cut(r))
            vp = self.radial_mlp(i, self.bessel_cut(r + eps))
            vm = self.radial_mlp(i, self.bessel_cut(r - eps))
        return dict(TV=v0, TG=(vp - vm) / (2.0 * eps) * h, h=h, M=M)

    def tp_weights(self, i: int, r: torch.Tensor, feats: torch.Tensor) -> torch.Tensor:
        """[E, nW*C] radial TP weights: the exact MLP, or the cubic Hermite interpolant of the fp64 table."""
        if self.tables is None:
            return self.radial_mlp(i, feats)
        t = self.tables[i]
        # x clamped to [0, M - 1 - 1e-4] (spline_w.py:19-27); the derivative is the interpolant's slope at the clamped
        # point times 1/h, also where x was clamped (r < r_lo): the reference's backward evaluates dW/dt at the clamped
        # t and scales it by inv_h unconditionally (spline_w.py:53-75, _w_bwd), so the clamp passes gradients through
        x = (r.reshape(-1) - self.r_lo) / t["h"]
        x = x.detach().clamp(0.0, t["M"] - 1 - 1e-4) + (x - x.detach())
        k = x.detach().floor().long()
        s = (x - k.to(x.dtype)).unsqueeze(-1)
        s2, s3 = s * s, s * s * s
        TV, TG = t["TV"], t["TG"]
        return ((2 * s3 - 3 * s2 + 1) * TV[k] + (s3 - 2 * s2 + s) * TG[k]
                + (-2 * s3 + 3 * s2) * TV[k + 1] + (s3 - s2) * TG[k + 1])

    # ------------------------------------------------------------------------------------------ building blocks
    def edge_embed(self, vec):
        r = torch.linalg.vector_norm(vec, dim=-1, keepdim=True)
        return r, sh_torch(vec), self.bessel_cut(r)

    def conv(self, i, X, Y, W, send, recv, n_out):
        """Channelwise TP summed on receivers.  X: list per node irrep of [n, C, 2l+1]; returns list per mid entry
        of [n_out, C, 2lo+1] (mid entries sorted by output l)."""
        nirr = [(0, 1)] if i == 0 else C_HIDDEN
        E = Y.shape[0]
        Wv = W.view(E, -1, self.C)
        out = []
        for w, (lo, i1, i2) in enumerate(self.inst[i]):
            l1 = nirr[i1][0]
            cg = self.w3[(l1, i2, lo)]
            xs = X[i1][send]                                             # [E, C, 2l1+1]
            m = torch.einsum("ecj,ek,jkm->ecm", xs, Y[:, _lsl(i2)], cg) * Wv[:, w, :].unsqueeze(-1)
            acc = torch.zeros(n_out, self.C, 2 * lo + 1, dtype=m.dtype)
            acc.index_add_(0, recv, m)
            out.append(acc)
        return out

    def linear_mid(self, i, mid):
        """e3nn Linear mid irreps -> 128x{0e,1o,2e,3o}: per output l sum over its mid copies, 1/sqrt(n_l C)."""
        W = self.P[f"interactions.{i}.linear.weight"]
        outs = []
        for l in range(4):
            ws = [w for w, (lo, _a, _b) in enumerate(self.inst[i]) if lo == l]
            acc = sum(torch.einsum("ncm,cd->ndm", mid[w], W[w]) for w in ws)
            outs.append(acc / math.sqrt(len(ws) * self.C))
        return outs

    def sym_contract(self, prefix, L, x, spec):
        """products.k symmetric contraction to irrep L: x [n, C, 16] -> [n, C, 2L+1]."""
        n = x.shape[0]
        out = torch.zeros(n, self.C, 2 * L + 1, dtype=x.dtype)
        for z in torch.unique(spec).tolist():
            sel = (spec == z).nonzero().flatten()
            for s0 in range(0, sel.numel(), 256):
                idx = sel[s0:s0 + 256]
                xs = x[idx]
                W = [self.P[f"{prefix}.sc.{L}.{nu}"][z] for nu in (1, 2, 3)]                 # [K, C]
                t3 = torch.einsum("Mijlk,kc->Mijlc", self.U[(L, 3)], W[2])
                o = torch.einsum("Mijlc,ncl->nMijc", t3, xs)
                o = o + torch.einsum("Mijk,kc->Mijc", self.U[(L, 2)], W[1]).unsqueeze(0)
                o = torch.einsum("nMijc,ncj->nMic", o, xs)
                o = o + torch.einsum("Mik,kc->Mic", self.U[(L, 1)], W[0]).unsqueeze(0)
                o = torch.einsum("nMic,nci->ncM", o, xs)
                out = out.index_put((idx,), o, accumulate=True)
        return out

    # ------------------------------------------------------------------------------------------ the two layers
    def layer1(self, vec, spec_nodes, send, recv, nC):
        """h1 [nC, C, 4] (0e | 1o) of the first nC nodes (the receivers); spec = model column per node."""
        C, Pm = self.C, self.P
        r, Y, feats = self.edge_embed(vec)
        emb = Pm["node_embedding.weight"][spec_nodes] / math.sqrt(self.Z)                 # [n, C]
        X = [(emb @ Pm["interactions.0.linear_up.weight"][0] / math.sqrt(C)).unsqueeze(-1)]
        W = self.tp_weights(0, r, feats)
        rho = torch.zeros(nC, 1, dtype=vec.dtype).index_add(0, recv, self.density(0, feats))
        mid = self.conv(0, X, Y, W, send, recv, nC)
        msg = self.linear_mid(0, mid)
        spec = spec_nodes[:nC]
        Ws = Pm["interactions.0.skip_tp.weight"]                                          # [4, C, Z, C]
        xl = []
        for l in range(4):
            m = msg[l] / (rho.unsqueeze(-1) + 1.0)
            xl.append(torch.einsum("ncm,ncd->ndm", m, Ws[l][:, spec, :].permute(1, 0, 2)) / math.sqrt(C * self.Z))
        x = torch.cat(xl, -1)                                                             # [nC, C, 16]
        A0 = self.sym_contract("products.0", 0, x, spec)
        A1 = self.sym_contract("products.0", 1, x, spec)
        Wp = Pm["products.0.linear.weight"]
        h0 = torch.einsum("ncm,cd->ndm", A0, Wp[0]) / math.sqrt(C)
        h1 = torch.einsum("ncm,cd->ndm", A1, Wp[1]) / math.sqrt(C)
        return torch.cat([h0, h1], -1)

    def readout1(self, h1):
        return (h1[:, :, 0] @ self.P["readouts.0.weight"]) / math.sqrt(self.C)

    def layer2_energy(self, vec, spec_nodes, h1_nodes, send, recv, nC):
        """Per-receiver R2 (unscaled) of the first nC nodes; h1_nodes [n, C, 4]."""
        C, Pm = self.C, self.P
        r, Y, feats = self.edge_embed(vec)
        spec = spec_nodes[:nC]
        Wsk = Pm["interactions.1.skip_tp.weight"][0]                                      # [C, Z, C]
        sc = torch.einsum("nc,ncd->nd", h1_nodes[:nC, :, 0], Wsk[:, spec, :].permute(1, 0, 2)) / math.sqrt(C * self.Z)
        Wu = Pm["interactions.1.linear_up.weight"]
        X = [torch.einsum("ncm,cd->ndm", h1_nodes[:, :, 0:1], Wu[0]) / math.sqrt(C),
             torch.einsum("ncm,cd->ndm", h1_nodes[:, :, 1:4], Wu[1]) / math.sqrt(C)]
        W = self.tp_weights(1, r, feats)
        rho = torch.zeros(nC, 1, dtype=vec.dtype).index_add(0, recv, self.density(1, feats))
        mid = self.conv(1, X, Y, W, send, recv, nC)
        msg = self.linear_mid(1, mid)
        x = torch.cat([m / (rho.unsqueeze(-1) + 1.0) for m in msg], -1)                   # [nC, C, 16]
        A = self.sym_contract("products.1", 0, x, spec)[:, :, 0]
        h2 = A @ Pm["products.1.linear.weight"][0] / math.sqrt(C) + sc
        z = h2 @ Pm["readouts.1.linear_1.weight"] / math.sqrt(C)
        a = self.cst * torch.nn.functional.silu(z)
        w2 = Pm["readouts.1.linear_2.weight"]
        return a @ w2 / math.sqrt(w2.shape[0])

    def e0(self, spec):
        return self.P["atomic_energies"][spec] + self.shift

    # ------------------------------------------------------------------------------------------ full graph
    def full_graph(self, pi, pj, rij, elems, nl, owner=None):
        """Energy per local atom and pair forces dE/drij by autograd over the whole graph (no chunking).
        pi receivers (local), pj senders (local or ghost), rij [P, 3] edge vectors, elems [nt] model columns,
        owner [nt] local owner of every atom (identity on locals) so that ghost rows carry their owner's h1."""
        pi, pj = torch.as_tensor(pi).long(), torch.as_tensor(pj).long()
        elems = torch.as_tensor(elems).long()
        nt = elems.numel()
        owner = torch.arange(nt) if owner is None else torch.as_tensor(owner).long()
        vec = torch.as_tensor(rij, dtype=torch.float64).clone().requires_grad_(True)
        h1 = self.layer1(vec, elems, pj, pi, nl)                                           # receivers = all locals
        R1 = self.readout1(h1)
        h1_nodes = h1[owner]
        R2 = self.layer2_energy(vec, elems, h1_nodes, pj, pi, nl)
        eat = self.e0(elems[:nl]) + self.scale * (R1 + R2)
        (gv,) = torch.autograd.grad(eat.sum(), [vec])
        return eat.detach(), gv.detach()

    # ------------------------------------------------------------------------------------------ three pass
    def three_pass(self, pi, pj, rij, elems, nl, chunk, owner=None, return_state=False, forward_exchange=None,
                   reverse_exchange=None):
        """The receiver-chunked three-pass evaluation with ML-IAP semantics; returns (eatoms [nl], PF [P, 3]) and,
        with return_state, also H1 [nt, C, 4] after the forward exchange and G1r [nl, C, 4] after the reverse one.
        forward_exchange / reverse_exchange (rows [nt, C*4], in place) replace the owner map, e.g. with the
        distributed halo exchange of a domain decomposition."""
        pi, pj = torch.as_tensor(pi).long(), torch.as_tensor(pj).long()
        elems = torch.as_tensor(elems).long()
        nt = elems.numel()
        owner = torch.arange(nt) if owner is None else torch.as_tensor(owner).long()
        rij = torch.as_tensor(rij, dtype=torch.float64)
        order = torch.argsort(pi, stable=True)
        pi_s, pj_s, rij_s = pi[order], pj[order], rij[order]
        rp = torch.searchsorted(pi_s, torch.arange(nl + 1))
        P = pi.numel()
        PF = torch.zeros(P, 3, dtype=torch.float64)
        eat = self.e0(elems[:nl]).clone()
        H1 = torch.zeros(nt, self.C, 4, dtype=torch.float64)
        bounds = [(a, min(a + chunk, nl)) for a in range(0, nl, chunk)]
        # pass A
        with torch.no_grad():
            for a, b in bounds:
                e0, e1 = int(rp[a]), int(rp[b])
                H1[a:b] = self._chunk_l1(a, b, e0, e1, pi_s, pj_s, rij_s, elems, None)
        if forward_exchange is not None:
            forward_exchange(H1.view(nt, -1))
        else:
            H1[nl:] = H1[owner[nl:]]                                                      # forward exchange
        # pass B
        G1 = torch.zeros_like(H1)
        for a, b in bounds:
            e0, e1 = int(rp[a]), int(rp[b])
            send = pj_s[e0:e1]
            outside = torch.unique(send[(send < a) | (send >= b)])
            nodes = torch.cat([torch.arange(a, b), outside])                                # receivers first
            loc = torch.full((nt,), -1, dtype=torch.long)
            loc[nodes] = torch.arange(nodes.numel())
            vec = rij_s[e0:e1].clone().requires_grad_(True)
            h1l = H1[nodes].clone().requires_grad_(True)
            R2 = self.layer2_energy(vec, elems[nodes], h1l, loc[send], pi_s[e0:e1] - a, b - a)
            eb = self.scale * R2.sum()
            gv, gh = torch.autograd.grad(eb, [vec, h1l])
            PF[order[e0:e1]] += gv
            G1.index_add_(0, nodes, gh)
            eat[a:b] += self.scale * R2.detach()
        if reverse_exchange is not None:
            G = G1.clone()
            reverse_exchange(G.view(nt, -1))
            G1r = G[:nl].clone()
        else:
            G1r = G1[:nl].clone()
            G1r.index_add_(0, owner[nl:], G1[nl:])                                        # reverse exchange
        # pass C
        for a, b in bounds:
            e0, e1 = int(rp[a]), int(rp[b])
            vec = rij_s[e0:e1].clone().requires_grad_(True)
            h1 = self._chunk_l1(a, b, e0, e1, pi_s, pj_s, rij_s, elems, vec)
            R1 = self.readout1(h1)
            loss = self.scale * R1.sum() + (G1r[a:b] * h1).sum()
            (gv,) = torch.autograd.grad(loss, [vec])
            PF[order[e0:e1]] += gv
            eat[a:b] += self.scale * R1.detach()
        if return_state:
            return eat, PF, H1, G1r
        return eat, PF

    def _chunk_l1(self, a, b, e0, e1, pi_s, pj_s, rij_s, elems, vec):
        send = pj_s[e0:e1]
        # layer-1 sender features depend only on the species: index senders directly, receivers 0..nC-1
        nodes = torch.cat([torch.arange(a, b), send])
        ls = torch.arange(b - a, b - a + send.numel())
        if vec is None:
            vec = rij_s[e0:e1]
        return self.layer1(vec, elems[nodes], ls, pi_s[e0:e1] - a, b - a)


def atom_forces(pi, pj, PF, nt):
    """F = -dE/dx from pair forces dE/dv with v = x_recv - x_send: F_recv -= PF, F_send += PF."""
    pi, pj = torch.as_tensor(pi).long(), torch.as_tensor(pj).long()
    F = torch.zeros(nt, 3, dtype=torch.float64)
    F.index_add_(0, pi, -PF)
    F.index_add_(0, pj, PF)
    return F
