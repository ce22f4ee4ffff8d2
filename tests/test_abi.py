"""The C-ABI library loads on a machine without a GPU and exports every entry point include/mace_b200.h declares;
the ctypes binding covers all of them (no compute calls here)."""
import ctypes
import os
import re

from mace_onegpu import _native as N

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mace_b200.h")


def declared():
    src = open(HDR).read()
    return sorted(set(re.findall(r"\b(mace_b200_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    names = declared()
    assert len(names) >= 20
    for nm in names:
        assert hasattr(lib, nm), nm
        assert nm in N.exported_symbols(), f"{nm} has no ctypes signature"


def test_struct_layouts_match_the_library():
    ms, es = N.c_i32(), N.c_i32()
    assert N.lib().mace_b200_struct_sizes(N.byref(ms), N.byref(es)) == 0
    assert ms.value == ctypes.sizeof(N.MBModel) and es.value == ctypes.sizeof(N.MBEval)
    assert N.MBModel.tab1.offset == 32 and N.MBEval.pair_i.offset == 16


def test_sc_layout_query():
    n = N.c_i32()
    fp = N.c_u64()
    assert N.lib().mace_b200_sc_layout(0, N.byref(n), N.byref(fp)) == 0 and n.value == 410
    assert N.lib().mace_b200_sc_layout(1, N.byref(n), N.byref(fp)) == 0 and n.value == 94
    assert N.lib().mace_b200_sc_layout(7, N.byref(n), N.byref(fp)) != 0
    assert b"block" in N.lib().mace_b200_last_error()


def test_hostio_cpulist_parsing():
    from mace_onegpu import hostio

    assert hostio._parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert hostio._parse_cpulist("") == set()


def test_custom_ops_register():
    """torch.ops.mace_b200: every custom op over the C ABI is registered with a schema (TORCH_LIBRARY), tensors and
    int64 / double / bool scalars only."""
    ops = N.ops()
    for name in N.OPS:
        schema = getattr(ops, name).default._schema
        assert schema.name == f"mace_b200::{name}"
        for arg in schema.arguments:
            assert str(arg.type) in ("Tensor", "Optional[Tensor]", "int", "float", "bool"), (name, arg)


def test_custom_op_errors_raise_runtime_error():
    """A failed check inside an op (TORCH_CHECK in the C++ wrapper) arrives in Python as RuntimeError with the
    reference's guard message (mliap_threepass.py:595-601), also for host tensors."""
    import pytest
    import torch

    ops = N.ops()
    ops.guard(torch.ones(4, dtype=torch.float64), 1.0, 100.0, 1)
    with pytest.raises(RuntimeError, match="non-finite or absurd output at call 2"):
        ops.guard(torch.ones(4, dtype=torch.float64), 250.0, 100.0, 2)
    with pytest.raises(RuntimeError, match="non-finite or absurd output"):
        ops.guard(torch.tensor([1.0, float("nan")], dtype=torch.float64), 1.0, 100.0, 3)
