"""Host-side guards of the ML-IAP wrapper that need no GPU.

The int32 neighbour-slot guard (reference mace_onegpu/mliap_threepass.py:450-461): LAMMPS' Kokkos neighbour list
indexes its slots with 32-bit ints, so a call whose pair count, grown by the skin shell, approaches 2^31 is refused
before any device work; MACE3P_ALLOW_HUGE=1 lifts the refusal.  The data object here only carries the sizes."""
import types

import pytest

from mace_onegpu import model as M
from mace_onegpu.mliap_threepass import ThreePassMLIAP


def _huge(npairs):
    return types.SimpleNamespace(nlocal=20_000_000, ntotal=24_000_000, npairs=npairs, elems=None)


@pytest.fixture(scope="module")
def mli():
    return ThreePassMLIAP(M.default_model(0), chunk=16384)


def test_int32_slot_guard_refuses_huge_pair_counts(mli, monkeypatch):
    monkeypatch.delenv("MACE3P_ALLOW_HUGE", raising=False)
    monkeypatch.setenv("MACE3P_SKIN", "2.0")
    # 1.2e9 pairs x ((6 + 2) / 6)^3 = 2.84e9 estimated slots > 0.95 * 2^31
    with pytest.raises(RuntimeError, match="2\\^31 int32 limit"):
        mli.compute_forces(_huge(1_200_000_000))


def test_int32_slot_guard_depends_on_the_skin(mli, monkeypatch):
    monkeypatch.delenv("MACE3P_ALLOW_HUGE", raising=False)
    monkeypatch.setenv("MACE3P_SKIN", "0.0")
    # without a skin 1.2e9 slots stay below the limit: the guard passes and the call reaches the data (elems=None)
    with pytest.raises((TypeError, RuntimeError, AttributeError)) as ei:
        mli.compute_forces(_huge(1_200_000_000))
    assert "int32 limit" not in str(ei.value)


def test_empty_calls_return_without_work(mli):
    mli.compute_forces(types.SimpleNamespace(nlocal=0, ntotal=0, npairs=0))
    mli.compute_forces(types.SimpleNamespace(nlocal=5, ntotal=5, npairs=1))
