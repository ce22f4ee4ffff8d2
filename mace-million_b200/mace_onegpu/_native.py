"""ctypes binding of libmace_b200.so (C ABI declared in include/mace_b200.h).

The structs below mirror mb_model_t / mb_eval_t field by field.  The library is loaded once; a missing library is
an error (there is no fallback implementation of any kernel).
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libmace_b200.so")

c_i32, c_i64, c_u32, c_u64, c_f32, c_f64 = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64,
                                            ctypes.c_float, ctypes.c_double)
c_vp = ctypes.c_void_p


ABI_VERSION = 4          # MB_ABI_VERSION of include/mace_b200.h this binding mirrors
ST_UNSORTED = 64         # MB_ST_UNSORTED


class MBModel(ctypes.Structure):
    _fields_ = [("C", c_i32), ("S", c_i32), ("M", c_i32),
                ("r_lo", c_f32), ("inv_h", c_f32), ("r_max", c_f32), ("p_cut", c_f32), ("scale", c_f32),
                ("tab1", c_vp), ("tab2", c_vp), ("wd1", c_vp), ("wd2", c_vp),
                ("M0", c_vp), ("M0T", c_vp), ("Wp1", c_vp), ("Wp1T", c_vp), ("wr0", c_vp), ("sc1", c_vp),
                ("Wup2", c_vp), ("Wup2T", c_vp), ("Wsk1", c_vp), ("Wsk1T", c_vp), ("Wlin2", c_vp), ("Wlin2T", c_vp),
                ("sc2", c_vp), ("Wp2", c_vp), ("Wp2T", c_vp), ("W1r", c_vp), ("w2r", c_vp), ("e0", c_vp),
                ("M0_tc", c_vp), ("M0T_tc", c_vp), ("Wp1_tc", c_vp), ("Wp1T_tc", c_vp), ("Wup2_tc", c_vp),
                ("Wup2T_tc", c_vp), ("Wsk1_tc", c_vp), ("Wsk1T_tc", c_vp), ("Wlin2_tc", c_vp), ("Wlin2T_tc", c_vp),
                ("Wp2_tc", c_vp), ("Wp2T_tc", c_vp), ("use_tc", c_i32), ("tab1_map", c_vp), ("tab2_map", c_vp),
                ("l1_density", c_i32)]


class MBEval(ctypes.Structure):
    _fields_ = [("nl", c_i32), ("nt", c_i32), ("P", c_i64),
                ("pair_i", c_vp), ("pair_j", c_vp), ("rij", c_vp), ("rowptr", c_vp), ("spec", c_vp),
                ("H1", c_vp), ("X2", c_vp), ("G1", c_vp), ("GX2", c_vp), ("PF", c_vp), ("eat", c_vp),
                ("chunk", c_i32), ("order", c_vp), ("spec_off", c_vp),
                ("s_msg", c_vp), ("s_x", c_vp), ("s_gx", c_vp), ("s_a", c_vp), ("s_ga", c_vp), ("s_h", c_vp),
                ("s_gh", c_vp), ("s_sc", c_vp), ("s_rho", c_vp), ("s_grho", c_vp), ("status", c_vp),
                ("x1_cache", c_vp), ("rho1_cache", c_vp), ("wait_ev", c_vp), ("done_ev", c_vp),
                ("pf_out", c_vp), ("fmax_bits", c_vp)]


_SIGS = {
    "mace_b200_abi_version": (c_i32, []),
    "mace_b200_last_error": (ctypes.c_char_p, []),
    "mace_b200_launch_count": (ctypes.c_ulonglong, []),
    "mace_b200_struct_sizes": (c_i32, [ctypes.POINTER(c_i32), ctypes.POINTER(c_i32)]),
    "mace_b200_timing": (c_i32, [c_i32, c_vp, c_vp]),
    "mace_b200_timing_kinds": (c_i32, [ctypes.c_uint32]),
    "mace_b200_ffma_peak": (c_i32, [c_i32, c_vp, c_vp, c_vp]),
    "mace_b200_sc_layout": (c_i32, [c_i32, ctypes.POINTER(c_i32), ctypes.POINTER(c_u64)]),
    "mace_b200_build_tables": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_i32, c_i32, c_f64, c_f64,
                                       c_f64, c_vp, c_vp, c_vp, c_vp]),
    "mace_b200_build_tables_noalloc": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_i32, c_i32, c_f64,
                                               c_f64, c_f64, c_vp, c_vp, c_vp, c_vp]),
    "mace_b200_edge_l1_fwd": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_edge_l2_fwd": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_edge_l2_bwd": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_edge_l1_bwd": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_conv_tp_fwd": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_vp, c_i32, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp,
                                      c_i32, c_vp, c_i32, c_vp, c_vp]),
    "mace_b200_conv_tp_bwd": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                      c_i32, c_vp, c_vp, c_i32, c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mace_b200_node_gemm": (c_i32, [c_vp, c_i64, c_vp, c_i32, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp, c_i32, c_vp,
                                    c_i32, c_vp]),
    "mace_b200_node_gemm_tc": (c_i32, [c_vp, c_i64, c_vp, c_i32, c_vp, c_i64, c_vp, c_i64, c_i32, c_i32, c_vp, c_i32,
                                       c_vp, c_i32, c_vp, c_vp]),
    "mace_b200_symcon_fwd": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_i32, c_vp]),
    "mace_b200_symcon_bwd": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_vp]),
    "mace_b200_pass_a": (c_i32, [c_vp, c_vp, c_vp]),
    "mace_b200_x2_all": (c_i32, [c_vp, c_vp, c_vp]),
    "mace_b200_pass_b": (c_i32, [c_vp, c_vp, c_vp]),
    "mace_b200_pass_c": (c_i32, [c_vp, c_vp, c_vp]),
    "mace_b200_finalize": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mace_b200_pass_a_chunks": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_x2_rows": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_pass_b_chunks": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_fold_g1": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_pass_c_chunks": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "mace_b200_pack_rows": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_vp, c_vp]),
    "mace_b200_unpack_add_rows": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_vp, c_vp]),
    "mace_b200_nbr_count": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_f64, c_vp, c_vp]),
    "mace_b200_nbr_fill": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_f64, c_vp, c_vp, c_vp,
                                   c_vp, c_vp, c_vp]),
    "mace_b200_verlet_filter": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_f64, c_vp, c_vp, c_vp, c_vp, c_vp,
                                        c_vp, c_vp]),
    "mace_b200_csr_rows": (c_i32, [c_vp, c_i64, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "mace_b200_sender_range": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_vp]),
    "mace_b200_tc_test_hooks": (c_i32, [c_u64, c_i32]),
}

_lib = None


def lib():
    """The loaded library (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python mace-million_b200/build.py` "
                               "(the CUDA path has no fallback implementation)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        abi = L.mace_b200_abi_version()
        if abi != ABI_VERSION:
            raise RuntimeError(f"libmace_b200.so ABI {abi} != {ABI_VERSION}: rebuild it with "
                               "`python mace-million_b200/build.py`")
        ms, es = c_i32(), c_i32()
        L.mace_b200_struct_sizes(ctypes.byref(ms), ctypes.byref(es))
        if (ms.value, es.value) != (ctypes.sizeof(MBModel), ctypes.sizeof(MBEval)):
            raise RuntimeError(f"libmace_b200.so struct sizes {ms.value}/{es.value} do not match the binding "
                               f"{ctypes.sizeof(MBModel)}/{ctypes.sizeof(MBEval)}")
        _lib = L
    return _lib


OPS_PATH = os.path.join(_HERE, "_lib", "libmace_b200_torch.so")
OPS = ("conv_tp", "conv_tp_backward", "build_tables", "edge_l1_fwd", "edge_l1_bwd", "edge_l2_fwd", "edge_l2_bwd",
       "node_gemm", "symcon_fwd", "symcon_bwd", "pack_halo", "unpack_halo_add", "csr_rows", "guard")
_ops = None


def ops():
    """torch.ops.mace_b200: the TORCH_LIBRARY custom ops of libmace_b200_torch.so over this library's C ABI (loaded
    once; raises if it was not built: there is no fallback)."""
    global _ops
    if _ops is None:
        import torch

        lib()
        if not os.path.exists(OPS_PATH):
            raise RuntimeError(f"{OPS_PATH} is missing: build it with `python mace-million_b200/build.py`")
        torch.ops.load_library(OPS_PATH)
        _ops = torch.ops.mace_b200
        _register_python_side(torch)
    return _ops


def _register_python_side(torch):
    """Shape functions (FakeTensor / meta) and the autograd formula of the ops that return new tensors."""
    from torch import library as tl

    @tl.register_fake("mace_b200::conv_tp")
    def _conv_fake(node_feats, edge_attrs, tp_weights, edge_index, terms, coef, n_out):
        return node_feats.new_empty((node_feats.shape[0], n_out * 128))

    @tl.register_fake("mace_b200::conv_tp_backward")
    def _conv_bwd_fake(grad, node_feats, edge_attrs, tp_weights, edge_index, terms, coef, n_out, nx, ny, nw):
        return (node_feats.new_empty(node_feats.shape), edge_attrs.new_empty(edge_attrs.shape),
                tp_weights.new_empty(tp_weights.shape))

    @tl.register_fake("mace_b200::pack_halo")
    def _pack_fake(src, idx):
        return src.new_empty((idx.shape[0], src.shape[1]))

    def _setup(ctx, inputs, output):
        node_feats, edge_attrs, tp_weights, edge_index, terms, coef, n_out = inputs
        ctx.save_for_backward(node_feats, edge_attrs, tp_weights, edge_index, terms, coef)
        ctx.n_out = n_out

    def _backward(ctx, grad):
        X, Y, W, ei, terms, coef = ctx.saved_tensors
        need = ctx.needs_input_grad
        dX, dY, dW = torch.ops.mace_b200.conv_tp_backward(grad.contiguous(), X, Y, W, ei, terms, coef, ctx.n_out,
                                                          bool(need[0]), bool(need[1]), bool(need[2]))
        return (dX if need[0] else None, dY if need[1] else None, dW if need[2] else None, None, None, None, None)

    tl.register_autograd("mace_b200::conv_tp", _backward, setup_context=_setup)


def exported_symbols():
    return list(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().mace_b200_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def ptr(t) -> int | None:
    """Device (or host) address of a tensor, None for None."""
    return None if t is None else int(t.data_ptr())


def byref(s):
    return ctypes.byref(s)


KINDS = ("edge_l1_fwd", "edge_l1_bwd", "edge_l2_fwd", "edge_l2_bwd", "symcon", "node_gemm")


def timing(enable: bool):
    """Collect (and reset) the per-kind kernel timings; switch recording on/off.  Returns {kind: (ms, launches)}."""
    ms = (ctypes.c_double * len(KINDS))()
    cnt = (ctypes.c_longlong * len(KINDS))()
    check(lib().mace_b200_timing(1 if enable else 0, ctypes.cast(ms, c_vp), ctypes.cast(cnt, c_vp)), "timing")
    return {k: (ms[i], cnt[i]) for i, k in enumerate(KINDS)}


def timing_kinds(kinds=None) -> None:
    """Record only these kinds (names of KINDS) while timing is on; None = all."""
    mask = 0xFFFFFFFF if kinds is None else sum(1 << KINDS.index(k) for k in kinds)
    check(lib().mace_b200_timing_kinds(mask), "timing_kinds")


def launch_count() -> int:
    return int(lib().mace_b200_launch_count())
