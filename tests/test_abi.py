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
