"""The tcgen05 3xTF32 node GEMM (mace_b200_node_gemm_tc) against the SIMT fp32 node GEMM (mace_b200_node_gemm) on
the row-gather shapes the passes use: multiplicities 1 / 3 / 5 / 7, 1-3 K segments, species-order gathers, the
1 / (rho + 1) row scale, accumulation, and row counts that are not multiples of the 128-row tile."""
import numpy as np
import pytest
import torch

from mace_onegpu import _native as N
from mace_onegpu import engine as E

pytestmark = pytest.mark.gpu
C = 128


def _run(tc, X, ldx, xoff, B, Y, ldy, yoff, mult, order, n, rho, acc):
    L = N.lib()
    st = torch.cuda.current_stream().cuda_stream
    xo = (N.c_i32 * 4)(*(list(xoff) + [0] * (4 - len(xoff))))
    if tc:
        Bt = torch.as_tensor(E.tc_planes(B.double().cpu().numpy()), device="cuda").contiguous()
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        N.check(L.mace_b200_node_gemm_tc(N.ptr(X), ldx, xo, len(xoff), N.ptr(Bt), Bt[0].numel(), N.ptr(Y), ldy, yoff,
                                         mult, N.ptr(order), n, N.ptr(rho), acc, N.ptr(status), st), "gemm_tc")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
    else:
        N.check(L.mace_b200_node_gemm(N.ptr(X), ldx, xo, len(xoff), N.ptr(B), N.ptr(Y), ldy, yoff, mult, N.ptr(order),
                                      n, N.ptr(rho), acc, st), "gemm")
        torch.cuda.synchronize()


@pytest.mark.parametrize("mult,xoff,ncomp,yoff,ycomp,n,use_order,use_rho,acc", [
    (1, [0], 4, 0, 4, 1000, False, False, 0),
    (3, [1], 4, 1, 4, 333, True, True, 1),
    (5, [4], 16, 4, 16, 129, True, True, 0),
    (7, [26, 33], 40, 9, 16, 517, False, True, 0),
    (3, [2, 5, 8], 40, 1, 16, 2048, False, True, 1),
    # more tiles than SMs: every persistent CTA runs several tiles, both TMEM accumulators and all stage phases wrap
    (3, [1], 4, 1, 4, 50000, True, True, 1),
    (1, [0, 2], 4, 1, 4, 70001, False, False, 0),
])
def test_tc_gemm_matches_simt(mult, xoff, ncomp, yoff, ycomp, n, use_order, use_rho, acc):
    g = torch.Generator(device="cuda").manual_seed(1)
    X = torch.randn(n, ncomp, C, device="cuda", generator=g)
    B = torch.randn(len(xoff), C, C, device="cuda", generator=g) / np.sqrt(C * len(xoff))
    order = torch.randperm(n, device="cuda", generator=g).to(torch.int32) if use_order else None
    rho = torch.rand(n, device="cuda", generator=g) * 3 if use_rho else None
    Y0 = torch.randn(n, ycomp, C, device="cuda", generator=g)
    Ys, Yt = Y0.clone(), Y0.clone()
    _run(False, X, ncomp * C, xoff, B.contiguous(), Ys, ycomp * C, yoff, mult, order, n, rho, acc)
    _run(True, X, ncomp * C, xoff, B.contiguous(), Yt, ycomp * C, yoff, mult, order, n, rho, acc)
    # 3xTF32 drops the lo*lo product (2^-22 relative per term); over K <= 384 random terms that stays < 1e-5 of the
    # output scale (TF32 alone would be ~1e-3)
    scale = Ys.abs().max().item()
    assert (Yt - Ys).abs().max().item() <= 1e-5 * scale


def test_tc_gemm_timeout_path_reports_and_recovers():
    """The bounded-wait error path, driven from the host: with one producer arrival withheld (test hook), the
    kernel's barrier waits expire after 20 ms, it drains its copies and MMAs, frees its TMEM and sets
    MB_ST_TC_TIMEOUT in the status word; the next launch with the default limit is correct."""
    L = N.lib()
    n, xoff = 3000, [0]
    g = torch.Generator(device="cuda").manual_seed(2)
    X = torch.randn(n, 1, C, device="cuda", generator=g)
    B = (torch.randn(1, C, C, device="cuda", generator=g) / np.sqrt(C)).contiguous()
    Bt = torch.as_tensor(E.tc_planes(B.double().cpu().numpy()), device="cuda").contiguous()
    st = torch.cuda.current_stream().cuda_stream
    xo = (N.c_i32 * 4)(0, 0, 0, 0)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    Y = torch.zeros(n, 1, C, device="cuda")
    try:
        N.check(L.mace_b200_tc_test_hooks(20_000_000, 1), "tc_test_hooks")
        N.check(L.mace_b200_node_gemm_tc(N.ptr(X), C, xo, 1, N.ptr(Bt), Bt[0].numel(), N.ptr(Y), C, 0, 1, None, n,
                                         None, 0, N.ptr(status), st), "gemm_tc")
        torch.cuda.synchronize()
        assert int(status.item()) & 32                       # MB_ST_TC_TIMEOUT
    finally:
        N.check(L.mace_b200_tc_test_hooks(2_000_000_000, 0), "tc_test_hooks")
    status.zero_()
    N.check(L.mace_b200_node_gemm_tc(N.ptr(X), C, xo, 1, N.ptr(Bt), Bt[0].numel(), N.ptr(Y), C, 0, 1, None, n, None,
                                     0, N.ptr(status), st), "gemm_tc")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = X[:, 0].double() @ B[0].double()
    assert (Y[:, 0].double() - want).abs().max().item() <= 1e-5 * want.abs().max().item()
