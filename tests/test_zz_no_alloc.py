"""The allocation-free table builder (mace_b200_build_tables_noalloc) against the allocating one.

Some callers cannot let a library allocate device memory (an MD engine that owns all device memory through its own
pool, or a process with a fixed device footprint); for them the library keeps the table builder's fp64 scratch in a
static device array.  This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.  It passes alone in a fresh process and after the other tests."""
import ctypes

import pytest
import torch

from mace_onegpu import _native as N
from mace_onegpu import engine as E
from mace_onegpu import model as M

pytestmark = pytest.mark.gpu

REL_TOL = 1e-6      # the tolerance of the table parity test (tests/test_gpu_parity.py)


def _inputs(layer, S=2, knots=512):
    mdl = M.default_model(0)
    f = E.fold_weights(mdl, [0, 7][:S])           # H and O columns
    A = [torch.as_tensor(x, dtype=torch.float64, device="cuda").contiguous() for x in f[f"A{layer}"]]
    cs = None
    if layer == 0:
        cs = torch.as_tensor(f["col_scale1"], dtype=torch.float64, device="cuda").contiguous()
    D = A[3].shape[1]
    return mdl, A, cs, D, S * S, knots


def _build(fn, mdl, A, cs, D, P, knots):
    TV = torch.full((P, knots, D), float("nan"), dtype=torch.float32, device="cuda")
    TG = torch.full_like(TV, float("nan"))
    cub = torch.full((P, knots - 1, D, 4), float("nan"), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = fn(N.ptr(A[0]), N.ptr(A[1]), N.ptr(A[2]), N.ptr(A[3]), A[0].shape[0], A[0].shape[1], D, N.ptr(cs), P, knots,
            0.5, float(mdl.arch.r_max), float(mdl.arch.num_poly_cutoff), N.ptr(TV), N.ptr(TG), N.ptr(cub), st)
    N.check(rc, fn.__name__)
    torch.cuda.synchronize()
    return TV, TG, cub


def _close(a, b):
    scale = b.abs().max().item() + 1e-30
    return bool(torch.isfinite(a).all()) and (a - b).abs().max().item() <= REL_TOL * scale


@pytest.mark.parametrize("layer", [0, 1])
def test_noalloc_tables_match_allocating_builder_twice(layer):
    L = N.lib()
    args = _inputs(layer)
    ref = _build(L.mace_b200_build_tables, *args)
    for _ in range(2):                           # two calls in a row share (and overwrite) the static scratch
        got = _build(L.mace_b200_build_tables_noalloc, *args)
        for g, r in zip(got, ref):
            assert _close(g, r)


def test_noalloc_rejects_tables_beyond_its_capacity():
    L = N.lib()
    mdl, A, cs, D, P, _ = _inputs(1)
    st = torch.cuda.current_stream().cuda_stream
    # null outputs: even if the capacity check stopped firing, the kernels skip null TV / TG / cubic (nothing written)
    rc = L.mace_b200_build_tables_noalloc(N.ptr(A[0]), N.ptr(A[1]), N.ptr(A[2]), N.ptr(A[3]), A[0].shape[0],
                                          A[0].shape[1], D, None, P, 1024, 0.5, 6.0, 5.0, None, None, None, st)
    assert rc != 0
    assert b"capacity" in ctypes.string_at(L.mace_b200_last_error())
