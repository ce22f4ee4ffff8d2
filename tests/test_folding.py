"""CPU check of the host-side folding (engine.fold_weights) and of the generated layouts it feeds: an fp64 emulation
of the folded forward computation (the algebra the CUDA kernels implement: X1 folded into the layer-1 weights,
M0 = linear o skip per species, grouped layer-2 linear, monomial-form symmetric contractions, TP term tables)
reproduces the oracle's per-atom energies."""
import dataclasses
import math

import numpy as np
import pytest
import torch

from mace_onegpu import engine as E
from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import o3
from mace_onegpu import structures as S
from oracle import mace_ref

C = 128


def _silu(z):
    return z / (1.0 + np.exp(-z))


def _hidden(A, f):
    h = f
    for W in A[:3]:
        h = _silu(h @ W)
    return h


def _mlp(A, f):
    return _hidden(A, f) @ A[3]


def _feats(r, arch):
    n = np.arange(1, arch.num_bessel + 1)
    x = r / arch.r_max
    p = arch.num_poly_cutoff
    env = (1 - (p + 1) * (p + 2) / 2 * x ** p + p * (p + 2) * x ** (p + 1) - p * (p + 1) / 2 * x ** (p + 2)) * (x < 1)
    return math.sqrt(2 / arch.r_max) * np.sin(n * np.pi / arch.r_max * r) / r * env


def _sc(coef, ents, x, spec, nout_base):
    """x [n, 16, C] -> out [n, nout, C] with per-(species, channel) monomial coefficients."""
    n = x.shape[0]
    nout = max(nout_base[L] + 2 * L + 1 for L in nout_base)
    out = np.zeros((n, nout, C))
    for t, (L, Mc, nu, mono, _row) in enumerate(ents):
        mo = np.ones((n, C))
        for i in mono:
            mo = mo * x[:, i, :]
        out[:, nout_base[L] + Mc, :] += coef[spec, t, :] * mo
    return out


def emulate(f, arch, pi, pj, rij, spec, nl, l1_density=False):
    t1, t2 = M.tp_tables()
    r = np.linalg.norm(rij, axis=1)
    Y = o3.sh_np(3, rij)
    feats = _feats(r[:, None], arch)
    S_ = f["S"]
    ss, sr = spec[pj], spec[pi]
    # layer 1
    rho1 = np.zeros(nl)
    np.add.at(rho1, pi, np.tanh((feats @ f["wd0"]) ** 2))
    if l1_density:
        # per-receiver densities B[m][slot H + q] of the MLP's hidden features, then the composite matrices
        hid = _hidden(f["A0"], feats)                                          # [E, H]
        H = hid.shape[1]
        msg1 = np.zeros((nl, 16, 2 * H))
        for mm in range(16):
            for s in range(S_):
                e = ss == s
                np.add.at(msg1[:, mm, s * H:(s + 1) * H], pi[e], hid[e] * Y[e, mm:mm + 1])
        M0 = E.fold_l1_density(f)
    else:
        W1 = _mlp(f["A0"], feats).reshape(-1, 4, C) * f["X1"][ss][:, None, :]
        msg1 = np.zeros((nl, 16, C))
        for l in range(4):
            for mm in range(l * l, (l + 1) ** 2):
                np.add.at(msg1[:, mm, :], pi, W1[:, l, :] * Y[:, mm:mm + 1])
        M0 = f["M0"]
    x1 = np.zeros((nl, 16, C))
    for l in range(4):
        sl = slice(l * l, (l + 1) ** 2)
        x1[:, sl, :] = np.einsum("nmc,ncd->nmd", msg1[:, sl, :], M0[spec[:nl], l]) / (rho1[:, None, None] + 1)
    A1 = _sc(f["sc0"], o3.sc_entries((0, 1)), x1, spec[:nl], {0: 0, 1: 1})
    h1 = np.zeros((nl, 4, C))
    h1[:, 0:1] = A1[:, 0:1] @ f["Wp1"][0]
    h1[:, 1:4] = A1[:, 1:4] @ f["Wp1"][1]
    R1 = h1[:, 0, :] @ f["wr0"]
    # layer 2 (nt == nl here)
    X2 = np.zeros_like(h1)
    X2[:, 0:1] = h1[:, 0:1] @ f["Wup2"][0]
    X2[:, 1:4] = h1[:, 1:4] @ f["Wup2"][1]
    W2 = _mlp(f["A1"], feats).reshape(-1, 10, C)
    rho2 = np.zeros(nl)
    np.add.at(rho2, pi, np.tanh((feats @ f["wd1"]) ** 2))
    msg2 = np.zeros((nl, 40, C))
    for (w, k, m, o, c) in t2["terms"]:
        np.add.at(msg2[:, o, :], pi, c * W2[:, w, :] * X2[pj, k, :] * Y[:, m:m + 1])
    offs = o3.mid_offsets(t2)
    x2 = np.zeros((nl, 16, C))
    for l, ws in t2["lin_groups"].items():
        for mm in range(2 * l + 1):
            x2[:, l * l + mm, :] = sum(msg2[:, offs[w] + mm, :] @ f["Wlin2"][w] for w in ws)
    x2 /= (rho2[:, None, None] + 1)
    A2 = _sc(f["sc1"], o3.sc_entries((0,)), x2, spec[:nl], {0: 0})[:, 0, :]
    sc = np.einsum("nc,ncd->nd", h1[:, 0, :], f["Wsk1"][spec[:nl]])
    h2 = sc + A2 @ f["Wp2"]
    R2 = _silu(h2 @ f["W1r"]) @ f["w2r"]
    return f["e0"][spec[:nl]] + arch.scale * (R1 + R2)


@pytest.mark.parametrize("l1_density", [False, True], ids=["direct", "density"])
def test_folded_forward_matches_oracle(l1_density):
    """Both layer-1 forms: W1 * X1 per edge (direct) and per-receiver hidden-feature densities mapped by the
    composite matrices of fold_l1_density (exact density projection)."""
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, seed=1)
    cols_all = S.species_columns(Z, mdl.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    cols = sorted(set(cols_all.tolist()))
    spec = np.array([cols.index(c) for c in cols_all])
    f = E.fold_weights(mdl, cols)
    assert E.l1_density_supported(f)
    e_emu = emulate(f, mdl.arch, pi.numpy().astype(np.int64), pj.numpy().astype(np.int64), rij.numpy(), spec, len(Z),
                    l1_density=l1_density)
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch))
    e_ref, _ = ref.three_pass(pi, pj, rij, cols_all, len(Z), 81)
    assert np.abs(e_emu - e_ref.numpy()).max() < 1e-9 * max(1.0, np.abs(e_ref.numpy()).max())


def test_density_layer1_needs_at_most_two_species():
    mdl = M.default_model(1)
    f = E.fold_weights(mdl, [0, 1, 2])
    assert not E.l1_density_supported(f)
    assert E.l1_density_supported(E.fold_weights(mdl, [5]))


def test_sc_layout_fingerprint_stable():
    # the generated kernels' coefficient order is fingerprinted; the host must reproduce it
    for Ls in ((0, 1), (0,)):
        ents = o3.sc_entries(Ls)
        assert o3.sc_fingerprint(ents) == o3.sc_fingerprint(o3.sc_entries(Ls))
    assert len(o3.sc_entries((0, 1))) == 410 and len(o3.sc_entries((0,))) == 94


def test_tc_planes_are_the_swizzled_split():
    """The tcgen05 B operand image: a permutation of each 128 x 128 matrix of the tf32 hi / lo split."""
    rng = np.random.default_rng(3)
    B = rng.normal(size=(3, 128, 128))
    pos = E.sw128_positions()
    assert sorted(pos.tolist()) == list(range(128 * 128))
    planes = E.tc_planes(B)
    split = E.tc_split(B)
    assert planes.shape == split.shape
    back = planes.reshape(-1, 128 * 128)[:, pos].reshape(split.shape)
    assert np.array_equal(back, split)


def test_dedup_tables_merges_only_identical():
    a = torch.randn(3, 5, 4, generator=torch.Generator().manual_seed(0))
    cub = torch.stack([a[0], a[1], a[0], a[2], a[1].clone()])
    cub[4, 2, 1] = torch.nextafter(cub[4, 2, 1], torch.tensor(float("inf")))   # one ulp apart: its own table
    t, m = E.dedup_tables(cub)
    assert m.tolist() == [0, 1, 0, 2, 3]
    assert t.shape[0] == 4
    for p in range(cub.shape[0]):
        assert torch.equal(t[m[p]], cub[p])


def test_tab2_pair_layout_is_the_documented_permutation():
    """[p][half][C] float4: half 0 = (a_2p, a_2p+1, b_2p, b_2p+1), half 1 = (c_2p, c_2p+1, d_2p, d_2p+1)."""
    T, K, nW = 2, 3, 10
    cub = torch.randn(T, K, nW * C, 4)
    out = E.tab2_pair_layout(cub)
    assert out.shape == cub.shape
    o = out.view(T, K, nW // 2, 2, C, 4)
    src = cub.view(T, K, nW, C, 4)
    for p in range(nW // 2):
        w0, w1 = 2 * p, 2 * p + 1
        assert torch.equal(o[:, :, p, 0], torch.stack([src[:, :, w0, :, 0], src[:, :, w1, :, 0],
                                                       src[:, :, w0, :, 1], src[:, :, w1, :, 1]], -1))
        assert torch.equal(o[:, :, p, 1], torch.stack([src[:, :, w0, :, 2], src[:, :, w1, :, 2],
                                                       src[:, :, w0, :, 3], src[:, :, w1, :, 3]], -1))
