"""The torch.ops.mace_b200 custom ops on the GPU.

* FusedConvTP (the reference's pickled fused-convolution module, mace_onegpu/fused_conv.py:20-37) through
  torch.ops.mace_b200.conv_tp and its registered autograd formula: forward and the three input gradients against the
  fp64 oracle's channelwise convolution (oracle/mace_ref.py MaceRef.conv, differentiated by torch autograd), for the
  layer-1 and layer-2 path tables, with edges in random order (the op groups them by receiver and by sender).
* build_tables against the C-ABI table builder; symcon_fwd / _bwd against direct C-ABI calls; node_gemm against
  torch; pack_halo / unpack_halo_add / csr_rows against torch indexing; the C-ABI sender_range against torch min / max;
  the output guard's RuntimeError."""
import dataclasses

import pytest
import torch

from mace_onegpu import _native as N
from mace_onegpu import engine as E
from mace_onegpu import model as M
from mace_onegpu.fused_conv import FusedConvTP
from oracle import mace_ref

pytestmark = pytest.mark.gpu

REL = 2e-5           # fp32 kernel against the fp64 oracle, relative to the largest magnitude


@pytest.fixture(scope="module")
def ref():
    mdl = M.default_model(0)
    return mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch))


def _close(a, b, rel=REL):
    a, b = a.double().cpu(), b.double().cpu()
    return (a - b).abs().max().item() <= rel * b.abs().max().item() + 1e-12


@pytest.mark.parametrize("layer", [0, 1])
def test_fused_conv_tp_matches_oracle(ref, layer):
    tab = M.tp_tables()[layer]
    nX, nW, nO, C = tab["nX"], tab["nW"], tab["nO"], 128
    n, E_ = 37, 600
    g = torch.Generator().manual_seed(layer)
    X = torch.randn(n, nX, C, generator=g, dtype=torch.float64)
    Y = torch.randn(E_, 16, generator=g, dtype=torch.float64)
    W = torch.randn(E_, nW * C, generator=g, dtype=torch.float64)
    snd = torch.randint(0, n, (E_,), generator=g)
    rcv = torch.randint(0, n, (E_,), generator=g)
    G = torch.randn(n, nO * C, generator=g, dtype=torch.float64)
    # oracle: X as a list per node irrep [n, C, 2l + 1], outputs per mid entry [n, C, 2lo + 1]
    Xr = X.clone().requires_grad_()
    Yr = Y.clone().requires_grad_()
    Wr = W.clone().requires_grad_()
    xs = [Xr[:, 0:1].permute(0, 2, 1)] + ([Xr[:, 1:4].permute(0, 2, 1)] if nX == 4 else [])
    outs = ref.conv(layer, xs, Yr, Wr, snd, rcv, n)
    want = torch.cat([o.permute(0, 2, 1) for o in outs], 1).reshape(n, nO * C)
    dX0, dY0, dW0 = torch.autograd.grad((want * G).sum(), [Xr, Yr, Wr])
    mod = FusedConvTP(tab, nW * C)
    dev = "cuda"
    Xd = X.reshape(n, nX * C).float().to(dev).requires_grad_()
    Yd = Y.float().to(dev).requires_grad_()
    Wd = W.float().to(dev).requires_grad_()
    out = mod(Xd, Yd, Wd, torch.stack([snd, rcv]).to(dev))
    assert _close(out, want)
    dX, dY, dW = torch.autograd.grad((out * G.float().to(dev)).sum(), [Xd, Yd, Wd])
    assert _close(dX, dX0.reshape(n, nX * C)) and _close(dY, dY0) and _close(dW, dW0)
    # deterministic: no atomics in the CSR kernels
    assert torch.equal(out, mod(Xd, Yd, Wd, torch.stack([snd, rcv]).to(dev)))


def test_build_tables_op_matches_c_abi():
    mdl = M.default_model(0)
    eng = E.ThreePassEngine(mdl, [0, 7], chunk=64, device="cuda", l1_mode="direct")
    A = eng.fm.t["_A1"]
    TV, TG, cub = N.ops().build_tables(A[0], A[1], A[2], A[3], None, 4, 512, 0.5, float(mdl.arch.r_max),
                                       float(mdl.arch.num_poly_cutoff))
    assert torch.equal(TV, eng.fm.TV[1]) and torch.equal(TG, eng.fm.TG[1])
    assert cub.shape == (4, 511, 1280, 4)


@pytest.mark.parametrize("block", [0, 1])
def test_symcon_ops_match_c_abi(block):
    mdl = M.default_model(0)
    eng = E.ThreePassEngine(mdl, [0, 7], chunk=64, device="cuda")
    sc = eng.fm.t["sc1" if block == 0 else "sc2"]
    n = 50
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(n, 16, 128, device="cuda", generator=g)
    spec = torch.randint(0, 2, (n,), device="cuda", dtype=torch.int32, generator=g)
    A = N.ops().symcon_fwd(sc, block, 2, x, spec)
    A0 = torch.empty_like(A)
    st = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().mace_b200_symcon_fwd(N.byref(eng.fm.struct), block, N.ptr(x), N.ptr(A0), N.ptr(spec), n, st),
            "symcon_fwd")
    assert torch.equal(A, A0)
    gA = torch.randn_like(A)
    rho = torch.rand(n, device="cuda", generator=g)
    gx, grho = N.ops().symcon_bwd(sc, block, 2, x, gA, spec, rho)
    gx0, grho0 = torch.empty_like(x), torch.empty_like(rho)
    N.check(N.lib().mace_b200_symcon_bwd(N.byref(eng.fm.struct), block, N.ptr(x), N.ptr(gA), N.ptr(gx0), N.ptr(spec),
                                         N.ptr(rho), N.ptr(grho0), n, st), "symcon_bwd")
    assert torch.equal(gx, gx0) and torch.equal(grho, grho0)


def test_node_gemm_op():
    g = torch.Generator(device="cuda").manual_seed(5)
    n = 300
    X = torch.randn(n, 4, 128, device="cuda", generator=g)
    B = torch.randn(2, 128, 128, device="cuda", generator=g) / 11.3
    Y = torch.zeros(n, 4, 128, device="cuda")
    rho = torch.rand(n, device="cuda", generator=g)
    xoff = torch.tensor([0, 1], dtype=torch.int32)
    N.ops().node_gemm(X, 512, xoff, B, Y, 512, 2, 1, None, n, rho, False)
    want = (X[:, 0] @ B[0] + X[:, 1] @ B[1]) / (rho[:, None] + 1.0)
    assert (Y[:, 2] - want).abs().max().item() < 1e-4
    assert Y[:, [0, 1, 3]].abs().max().item() == 0.0


def test_halo_pack_unpack_and_csr_rows_ops():
    ops = N.ops()
    g = torch.Generator(device="cuda").manual_seed(7)
    src = torch.randn(100, 512, device="cuda", generator=g)
    idx = torch.randint(0, 100, (40,), device="cuda", dtype=torch.int32, generator=g)
    buf = ops.pack_halo(src, idx)
    assert torch.equal(buf, src[idx.long()])
    dst = torch.zeros(100, 512, device="cuda")
    ops.unpack_halo_add(dst, buf, idx)
    want = torch.zeros(100, 512, device="cuda").index_add_(0, idx.long(), buf)
    assert (dst - want).abs().max().item() < 1e-5
    pi = torch.sort(torch.randint(0, 50, (1000,), device="cuda", generator=g)).values.to(torch.int32)
    rowptr = torch.full((51,), -1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    e25 = int(torch.searchsorted(pi, torch.tensor([25], dtype=torch.int32, device="cuda")).item())
    ops.csr_rows(pi, 0, e25, 0, 25, rowptr, status)
    ops.csr_rows(pi, e25, 1000, 25, 50, rowptr, status)
    want_rp = torch.searchsorted(pi, torch.arange(51, dtype=torch.int32, device="cuda")).to(torch.int32)
    assert torch.equal(rowptr, want_rp)
    assert int(status.item()) == 0
    ops.csr_rows(pi.flip(0).contiguous(), 0, 1000, 0, 50, rowptr, status)     # not sorted: flagged
    assert int(status.item()) == 64


def test_sender_range():
    """mace_b200_sender_range: (min, max) of pair_j over an edge range, (INT32_MAX, -1) for an empty range."""
    L = N.lib()
    g = torch.Generator(device="cuda").manual_seed(8)
    pj = torch.randint(0, 1_000_000, (3_000_000,), device="cuda", dtype=torch.int32, generator=g)
    out = torch.zeros(4, 2, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    cases = [(0, 3_000_000), (5, 6), (1_234_567, 2_500_001), (10, 10)]
    for q, (e0, e1) in enumerate(cases):
        N.check(L.mace_b200_sender_range(N.ptr(pj), e0, e1, N.ptr(out[q]), st), "sender_range")
    torch.cuda.synchronize()
    for q, (e0, e1) in enumerate(cases[:3]):
        assert out[q].tolist() == [int(pj[e0:e1].min()), int(pj[e0:e1].max())]
    assert out[3].tolist() == [2**31 - 1, -1]


def test_guard_op():
    ops = N.ops()
    eat = torch.ones(10, dtype=torch.float64, device="cuda")
    ops.guard(eat, 1.0, 100.0, 1)
    with pytest.raises(RuntimeError, match="non-finite or absurd output"):
        ops.guard(eat, 150.0, 100.0, 2)
    eat[3] = float("nan")
    with pytest.raises(RuntimeError, match="non-finite or absurd output"):
        ops.guard(eat, 1.0, 100.0, 3)


@pytest.mark.parametrize("l1_mode", ["density", "direct"])
def test_edge_ops_match_c_abi(l1_mode):
    """The four edge ops, given the engine's tensors, reproduce the C-ABI kernels called with the engine's structs
    (the op wrappers fill exactly the struct fields the kernels read)."""
    from mace_onegpu import neighbors as NB
    from mace_onegpu import structures as S

    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, seed=0)
    cols = torch.as_tensor(S.species_columns(Z, mdl.arch.atomic_numbers))
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    n = len(Z)
    eng = E.ThreePassEngine(mdl, sorted(set(cols.tolist())), chunk=n, device="cuda", l1_mode=l1_mode)
    plan = eng.plan(pi, pj, rij, cols.cuda(), n, n)
    eng.evaluate(plan)                                  # fills H1, X2 of the engine's buffers
    ev, b = eng.eval_struct(plan)
    L, ops, t = N.lib(), N.ops(), eng.fm.t
    st = torch.cuda.current_stream().cuda_stream
    m = N.byref(eng.fm.struct)
    geo = dict(S=eng.fm.S, M=eng.fm.M, r_lo=eng.fm.r_lo, r_max=eng.fm.r_max, p_cut=float(mdl.arch.num_poly_cutoff))
    pair = (plan.pi, plan.pj, plan.rij, plan.rowptr, plan.spec)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(11)
    # layer 2 forward
    N.check(L.mace_b200_edge_l2_fwd(m, N.byref(ev), 0, n, st), "edge_l2_fwd")
    msg0, rho0 = b["s_msg"][:n].clone(), b["s_rho"][:n].clone()
    msg, rho = torch.zeros_like(b["s_msg"]), torch.zeros_like(b["s_rho"])
    ops.edge_l2_fwd(t["tab2"], t["tab2_map"], t["wd2"], *pair, b["X2"], msg, rho, status, 0, n, **geo)
    assert torch.equal(msg[:n], msg0) and torch.equal(rho[:n], rho0)
    # layer 2 backward (dE/dX2 accumulates with atomics: equal to fp32 summation order)
    gmsg = torch.randn(b["s_msg"].shape, device="cuda", generator=g)
    grho = torch.randn(b["s_grho"].shape, device="cuda", generator=g)
    b["s_msg"].copy_(gmsg)
    b["s_grho"].copy_(grho)
    b["PF"].zero_()
    b["GX2"].zero_()
    N.check(L.mace_b200_edge_l2_bwd(m, N.byref(ev), 0, n, st), "edge_l2_bwd")
    PF0, GX0 = b["PF"].clone(), b["GX2"].clone()
    PF, GX = torch.zeros_like(PF0), torch.zeros_like(GX0)
    ops.edge_l2_bwd(t["tab2"], t["tab2_map"], t["wd2"], *pair, b["X2"], gmsg, grho, GX, PF, status, 0, n, **geo)
    assert torch.equal(PF, PF0) and _close(GX, GX0, 1e-6)
    # layer 1 forward / backward in the engine's form
    l1d = 1 if eng.fm.l1_density else 0
    N.check(L.mace_b200_edge_l1_fwd(m, N.byref(ev), 0, n, st), "edge_l1_fwd")
    msg1 = b["s_msg"].view(-1)[: n * 16 * 128].clone()            # layer-1 rows: [n][16][128] at the front
    rho1 = b["s_rho"][:n].clone()
    out, outr = torch.zeros(n * 16 * 128, device="cuda"), torch.zeros(n, device="cuda")
    ops.edge_l1_fwd(t["tab1"], t["tab1_map"], t["wd1"], l1d, *pair, out, outr, status, 0, n, **geo)
    assert torch.equal(out, msg1) and torch.equal(outr, rho1)
    g1 = torch.randn(n * 16 * 128, device="cuda", generator=g)
    b["s_msg"].view(-1)[: n * 16 * 128].copy_(g1)
    b["PF"].zero_()
    N.check(L.mace_b200_edge_l1_bwd(m, N.byref(ev), 0, n, st), "edge_l1_bwd")
    PF0 = b["PF"].clone()
    PF = torch.zeros_like(PF0)
    ops.edge_l1_bwd(t["tab1"], t["tab1_map"], t["wd1"], l1d, *pair, g1, b["s_grho"], PF, status, 0, n, **geo)
    assert torch.equal(PF, PF0)
    assert int(status.item()) == 0
