"""LAMMPS ML-IAP ("pair_style mliap unified <file.pt> 0") wrapper of the B200 three-pass MACE force evaluation.

Drop-in for the reference's ``mace_onegpu.mliap_threepass.ThreePassMLIAP`` (mace_onegpu/mliap_threepass.py:155-622):
same module path (pickles made with either resolve to this class), constructor signature, ML-IAP attributes,
``compute_forces(data)`` contract (per-atom energies into data.eatoms, data.energy, pair forces dE/drij through
data.update_pair_forces_gpu in the caller's pair order), H1 forward / G1 reverse exchange through
data.forward_exchange / data.reverse_exchange with the same 2^31-element column split, the same guards
(int32 neighbour-slot estimate, non-finite / absurd force abort) and the same MACE3P_* environment knobs that still
mean something (CHUNK, LOG, SKIN, ALLOW_HUGE, FMAX_ABORT, GRAPHS).

Per call: pass A (layer-1 features of every local atom) -> forward exchange -> pass B (layer-2 energy, pair forces,
G1 = dE2/dh1) -> reverse exchange -> pass C (loss E1 + G1 . h1, remaining pair forces); all arithmetic runs in the
sm_100a kernels of libmace_b200.so (engine.py), there is no other implementation.
"""
from __future__ import annotations

import json
import os
import time

import torch

from . import _native as N

try:
    from lammps.mliap.mliap_unified_abc import MLIAPUnified
except ImportError:  # pragma: no cover - LAMMPS is not part of this package
    class MLIAPUnified:
        def __init__(self):
            pass

_RUNTIME = ("_eng", "_dev", "_cols", "_log", "_fmax_abort", "_t_end")
_INT_MAX = 2 ** 31 - 1


def exchange_blocks(nt: int, D: int):
    """Column blocks (first column, width) of one exchange of an [nt, D] feature array.  LAMMPS' ML-IAP comm
    buffers are sized with 32-bit ints (ntotal * D), so every callback must move fewer than 2^31 - 1 elements: the
    width is D >> k for the smallest k that satisfies this (at least 1 column), the blocks tile [0, D) in order and
    the last one may be narrower.  This is the call pattern of the reference's _exchange
    (mace_onegpu/mliap_threepass.py:40-55), which halves the width until it fits."""
    if nt * D < _INT_MAX:
        return [(0, D)]
    k = 0
    while (D >> k) > 1 and nt * (D >> k) >= _INT_MAX:
        k += 1
    w = D >> k
    return [(c0, min(w, D - c0)) for c0 in range(0, D, w)]


def _exchange(fn, src, dst, D):
    """dst = fn applied to src, one callback per column block of exchange_blocks (blocks narrower than D go through
    contiguous copies: the callback sees a dense [nt, width] array)."""
    blocks = exchange_blocks(int(src.shape[0]), D)
    if len(blocks) == 1:
        fn(src, dst, D)
        return
    for c0, w in blocks:
        part_in = src[:, c0:c0 + w].contiguous()
        part_out = torch.empty_like(part_in)
        fn(part_in, part_out, w)
        dst[:, c0:c0 + w] = part_out


def neighbour_slot_guard(nl: int, P: int, r_max: float):
    """Refuse a call whose LAMMPS neighbour list would approach 2^31 slots (mace_onegpu/mliap_threepass.py:450-461):
    Kokkos indexes the full list, pairs inside r_max grown by the skin shell, with 32-bit ints, and an overflow there
    is an illegal device access inside LAMMPS.  Estimate P ((r_max + skin) / r_max)^3 against 0.95 * 2^31, skin from
    MACE3P_SKIN (2 A); MACE3P_ALLOW_HUGE=1 lifts the refusal.  The message is the reference's."""
    if os.environ.get("MACE3P_ALLOW_HUGE", "0") == "1":
        return
    skin = float(os.environ.get("MACE3P_SKIN", "2.0"))
    est_slots = P * ((r_max + skin) / r_max) ** 3
    if est_slots > 0.95 * 2 ** 31:
        raise RuntimeError(f"ThreePassMLIAP guard: nlocal={nl:,}, pairs={P:,} -> estimated LAMMPS neighbour slots "
                           f"{est_slots:.3e} is close to the 2^31 int32 limit of the Kokkos neighbour list "
                           f"(skin {skin} A). Use fewer atoms per GPU, a smaller skin, or more GPUs.")


class ThreePassMLIAP(MLIAPUnified):
    def __init__(self, model, chunk=16384, spline_grid=512, node_bucket=8192, e_align=65536, rebuild_config=None):
        super().__init__()
        from .model import CHEMICAL_SYMBOLS

        self.model = model
        self.element_types = [CHEMICAL_SYMBOLS[int(z)] for z in model.atomic_numbers]
        self.num_species = len(self.element_types)
        self.rcutfac = 0.5 * float(model.r_max)
        self.ndescriptors = 1
        self.nparams = 1
        self.chunk = int(chunk)
        self.spline_grid = int(spline_grid)
        # node_bucket / e_align pad the reference's cuEquivariance shapes; the B200 kernels need no padding
        self.node_bucket = int(node_bucket)
        self.e_align = int(e_align)
        self.dtype = torch.float32
        self.step = 0
        self._rebuild = None

    def __getstate__(self):
        d = self.__dict__.copy()
        for k in _RUNTIME:
            d.pop(k, None)
        return d

    # ------------------------------------------------------------------------------------------------ setup
    def _setup(self, elems):
        from .engine import ThreePassEngine

        dev = elems.device if elems.is_cuda else torch.device("cuda", torch.cuda.current_device())
        self._dev = dev
        if os.environ.get("MACE3P_CHUNK"):
            self.chunk = int(os.environ["MACE3P_CHUNK"])
        cols = sorted(int(c) for c in torch.unique(elems.long()).tolist())
        self._cols = cols
        self._eng = ThreePassEngine(self.model, cols, chunk=self.chunk, spline_grid=self.spline_grid or 512,
                                    device=dev)
        # MACE3P_GRAPHS=1 (mliap_threepass.py:255): replay the evaluation as one CUDA graph; the engine captures only
        # when no exchange has to run between the passes (one rank without ghosts)
        if os.environ.get("MACE3P_GRAPHS", "0") == "1":
            self._eng.graphs = True
        self._fmax_abort = float(os.environ.get("MACE3P_FMAX_ABORT", "100.0"))
        path = os.environ.get("MACE3P_LOG")
        self._log = open(path, "a", buffering=1) if path else None
        self._eng.pass_timing = self._log is not None

    # ------------------------------------------------------------------------------------------------ entry point
    def compute_forces(self, data):
        nl, nt, P = int(data.nlocal), int(data.ntotal), int(data.npairs)
        if nl == 0 or P <= 1:
            return
        t_start = time.perf_counter()
        prev_end = getattr(self, "_t_end", None)        # LAMMPS' time between two calls, for the per-call log
        neighbour_slot_guard(nl, P, 2.0 * self.rcutfac)
        elems = torch.as_tensor(data.elems)
        if not hasattr(self, "_eng"):
            self._setup(elems)
        self.step += 1
        # pinned host pair arrays stay on the host: the engine streams them in chunk by chunk during pass A
        pi, pj, rij = (torch.as_tensor(x) for x in (data.pair_i, data.pair_j, data.rij))
        try:
            plan = self._eng.plan(pi, pj, rij, elems.to(self._dev, non_blocking=True), nl, nt)
        except RuntimeError as err:
            if "has no tables" not in str(err):
                raise
            self._setup(elems)                      # a species appeared that the tables were not built for
            plan = self._eng.plan(pi, pj, rij, elems.to(self._dev, non_blocking=True), nl, nt)
        eng = self._eng
        t_prep = time.perf_counter() - t_start
        hbuf = getattr(data, "pair_forces_host", None)
        D = 512

        def fwd(H):
            tmp = torch.empty_like(H)
            _exchange(data.forward_exchange, H, tmp, D)
            H.copy_(tmp)

        def rev(G):
            tmp = torch.empty_like(G)
            _exchange(data.reverse_exchange, G, tmp, D)
            G.copy_(tmp)

        eat, PF = eng.evaluate(plan, fwd if nt > nl else None, rev if nt > nl else None, host_pf=hbuf)
        fmax = eng.fmax
        # force guard (mliap_threepass.py:595-601): torch.ops.mace_b200.guard raises RuntimeError on non-finite
        # energies or a pair-force maximum that is non-finite or not below MACE3P_FMAX_ABORT
        N.ops().guard(eat, float(fmax), float(self._fmax_abort), int(self.step))
        torch.as_tensor(data.eatoms).copy_(eat)
        data.energy = float(eat.sum())
        data.update_pair_forces_gpu(hbuf if eng.host_pf_written else PF)
        if self._log is not None:
            torch.cuda.synchronize()
            peak = torch.cuda.max_memory_allocated(self._dev) / 1e9
            torch.cuda.reset_peak_memory_stats(self._dev)
            self._log.write(json.dumps(dict(step=self.step, nlocal=nl, ntotal=nt, npairs=P,
                                            chunks=(nl + self.chunk - 1) // self.chunk,
                                            sorted_pairs=plan.perm is None, streamed_pairs=plan.host_src is not None,
                                            graphs=bool(eng.graphs), captures=eng.captures,
                                            t_total=time.perf_counter() - t_start, t_prep=t_prep, **eng.pass_times(),
                                            t_gap_lammps=None if prev_end is None else t_start - prev_end,
                                            peak_gb=peak, fmax=fmax)) + "\n")
        self._t_end = time.perf_counter()

    def compute_descriptors(self, data):
        pass

    def compute_gradients(self, data):
        pass
