#!/usr/bin/env python
"""Generate symcon_gen.cuh: unrolled per-(atom, channel) symmetric-contraction polynomials (correlation 3, l <= 3
inputs) for the two product blocks of the MACE-MPA-0 architecture, forward and backward.

    python mace-million_b200/csrc/gen_symcon.py        (rewrites csrc/symcon_gen.cuh)

The polynomial of output component (L, M) for one channel is sum_t coef[t] * mono_t(x) over the entries of
mace_onegpu.o3.sc_entries (canonical order); coef[t] is per species and channel, folded on the host and stored as
[species][t / 4][channel][t % 4] (engine.sc_coef_layout), so that one 16-byte load per thread brings the next four
coefficients (the code consumes t in increasing order).  The functions take K atoms of one species: each
coefficient is loaded once per call and applied to all K atoms.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from mace_onegpu import o3  # noqa: E402

BLOCKS = {0: (0, 1), 1: (0,)}


def gen_block(b, Ls):
    ents = o3.sc_entries(Ls)
    base = {}
    off = 0
    for L in Ls:
        base[L] = off
        off += 2 * L + 1
    nout = off
    fp = o3.sc_fingerprint(ents)
    # group consecutive entries by monomial
    groups = []
    for t, (L, M, nu, mono, _r) in enumerate(ents):
        key = (L, nu, mono)
        if groups and groups[-1][0] == key:
            groups[-1][1].append((t, base[L] + M))
        else:
            groups.append((key, [(t, base[L] + M)]))
    F, B = [], []
    # K atoms of one species per call: every coefficient is loaded once and applied to the K atoms' monomials
    F.append(f"template <int K>")
    F.append(f"__device__ __forceinline__ void sc{b}_fwd(const float (&x)[K][16], const float4* __restrict__ cf, "
             f"float (&out)[K][{nout}]) {{")
    F.append(f"  #pragma unroll\n  for (int a = 0; a < K; ++a)\n    #pragma unroll\n    for (int q = 0; q < {nout}; ++q) out[a][q] = 0.f;")
    F.append("  float pij[K], mo[K];\n  float c;\n  float4 c4;")
    B.append(f"template <int K>")
    B.append(f"__device__ __forceinline__ void sc{b}_bwd(const float (&x)[K][16], const float4* __restrict__ cf, "
             f"const float (&gA)[K][{nout}], float (&gx)[K][16]) {{")
    B.append("  #pragma unroll\n  for (int a = 0; a < K; ++a)\n    #pragma unroll\n    for (int q = 0; q < 16; ++q) gx[a][q] = 0.f;")
    B.append("  float pij[K], G[K];\n  float c;\n  float4 c4;")
    A = "  #pragma unroll\n  for (int a = 0; a < K; ++a) "

    def coef(t):
        """Coefficient t into c: a 16-byte load of t .. t + 3 when t % 4 == 0, then the component."""
        out = [f"  c4 = __ldg(cf + {t // 4} * MB_C);"] if t % 4 == 0 else []
        out.append(f"  c = c4.{'xyzw'[t % 4]};")
        return out

    def grad_sum(lst):
        # G[a] = sum over the group's (t, q) of gA[a][q] * cf_t, one coefficient load per entry
        out = []
        for n_, (t, q) in enumerate(lst):
            out += coef(t)
            out.append(A + (f"G[a] = gA[a][{q}] * c;" if n_ == 0 else f"G[a] = fmaf(gA[a][{q}], c, G[a]);"))
        return out

    prev_pair = None
    for (L, nu, mono), lst in groups:
        if nu == 1:
            (i,) = mono
            for t, q in lst:
                F += coef(t)
                F.append(A + f"out[a][{q}] = fmaf(c, x[a][{i}], out[a][{q}]);")
            B += grad_sum(lst)
            B.append(A + f"gx[a][{i}] += G[a];")
            continue
        if nu == 2:
            i, j = mono
            F.append(A + f"mo[a] = x[a][{i}] * x[a][{j}];")
            for t, q in lst:
                F += coef(t)
                F.append(A + f"out[a][{q}] = fmaf(c, mo[a], out[a][{q}]);")
            B += grad_sum(lst)
            if i == j:
                B.append(A + f"gx[a][{i}] = fmaf(2.f * G[a], x[a][{i}], gx[a][{i}]);")
            else:
                B.append(A + f"{{ gx[a][{i}] = fmaf(G[a], x[a][{j}], gx[a][{i}]); "
                             f"gx[a][{j}] = fmaf(G[a], x[a][{i}], gx[a][{j}]); }}")
            continue
        i, j, k = mono
        if prev_pair != (i, j):
            F.append(A + f"pij[a] = x[a][{i}] * x[a][{j}];")
            B.append(A + f"pij[a] = x[a][{i}] * x[a][{j}];")
            prev_pair = (i, j)
        F.append(A + f"mo[a] = pij[a] * x[a][{k}];")
        for t, q in lst:
            F += coef(t)
            F.append(A + f"out[a][{q}] = fmaf(c, mo[a], out[a][{q}]);")
        B += grad_sum(lst)
        # d/dx of x_i x_j x_k with i <= j <= k
        B.append(A + f"{{ gx[a][{k}] = fmaf(G[a], pij[a], gx[a][{k}]); const float Gk = G[a] * x[a][{k}]; "
                     f"gx[a][{i}] = fmaf(Gk, x[a][{j}], gx[a][{i}]); gx[a][{j}] = fmaf(Gk, x[a][{i}], gx[a][{j}]); }}")
    F.append("}")
    B.append("}")
    ts = [t for (_k, lst) in groups for (t, _q) in lst]
    assert ts == sorted(ts) == list(range(len(ents))), "coefficients must be consumed in increasing order"
    hdr = [f"#define SC{b}_NT {len(ents)}", f"#define SC{b}_NT4 {(len(ents) + 3) // 4}", f"#define SC{b}_NOUT {nout}",
           f"#define SC{b}_FP 0x{fp:016x}ull"]
    return hdr, F, B


def main():
    out = ["// GENERATED by csrc/gen_symcon.py from mace_onegpu.o3.sc_entries -- do not edit.",
           "// Symmetric contraction (correlation 3) of one channel: out[L,M] = sum_t coef_t * mono_t(x), coef_t = cf[t/4][C].(t%4).", "#pragma once", ""]
    bodies = []
    for b, Ls in BLOCKS.items():
        hdr, F, B = gen_block(b, Ls)
        out += hdr
        bodies += F + [""] + B + [""]
    out += ["", "namespace mb {"] + bodies + ["}  // namespace mb", ""]
    with open(os.path.join(HERE, "symcon_gen.cuh"), "w") as fh:
        fh.write("\n".join(out))


if __name__ == "__main__":
    main()
