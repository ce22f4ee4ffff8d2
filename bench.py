#!/usr/bin/env python
"""Force-evaluation throughput of the B200 three-pass MACE (the BASELINE metric: atoms/s per force evaluation on the
1.03M-atom water box, plus the roofline fraction of the dominant kernel).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config water_1m]

A step is one full force evaluation (pass A, H1 exchange, pass B, G1 exchange, pass C, output) of the configuration's
synthetic structure with random-init weights (seed 0; no dataset or checkpoint is used).  `value` times steps on
inputs already resident in HBM (the pair list is 2.2 GB of fp64 vectors, larger than L2, so no explicit flush);
`e2e` times the reference-facing call ThreePassMLIAP.compute_forces(data) with pinned host buffers, the host->device
copies of the pair list and the device->host copies of energies and pair forces inside the timed region.
`--impl reference` times the CPU fp64 restatement of the reference's algorithm (oracle/, the reference itself cannot
be installed: mace-torch / e3nn / cuEquivariance are absent) on a bounded sample of the same workload.
Multi-GPU (torchrun, one rank per GPU): spatial domain decomposition of the periodic box (2x1x1, 2x2x1, 2x2x2 blocks)
with explicit ghost atoms (shell r_max + 2 A skin) and the H1 forward / G1 reverse halo exchanges as NCCL grouped
send/recv inside every timed step.  --scaling weak (default) keeps 1.03M atoms per GPU (the global box grows with N,
BASELINE config 5 at N = 8); --scaling strong splits the 1.03M-atom box over the N GPUs.  The decomposition is
built on the GPU (domain.DeviceDecomposition).  `md` times --md-steps velocity-Verlet steps of the same box at every
N (one GPU: md.VelocityVerlet; N GPUs: md.DomainVelocityVerlet on the same domains).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "mace-million_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "force-eval atoms/sec at 1.03M-atom water, 1/2/4/8 B200; % of HBM/TC roofline"
CONFIGS = {
    "water_1m": dict(kind="water", n=70, seed=0, model_seed=0,
                     desc="1,029,000-atom water box: 343,000 H2O on a 70^3 grid spaced 3.104 A (box 217.28 A)"),
    "water_24k": dict(kind="water", n=20, seed=0, model_seed=0, desc="24,000-atom water box (20^3 H2O)"),
    "water_192": dict(kind="water", n=4, seed=0, model_seed=0, desc="192-atom water box (4^3 H2O)"),
    "alloy_432k": dict(kind="alloy", n=60, seed=0, model_seed=1, desc="432,000-atom 16-element bcc alloy"),
    "water_8m": dict(kind="water", n=140, seed=0, model_seed=0,
                     desc="8,232,000-atom water box on one GPU (140^3 H2O, BASELINE config 5's box): memory scaling"),
}
# Algorithmic FLOPs per edge of each edge kernel, counted from the algorithm (C = 128 channels, 86 / 16 CG terms,
# 10 / 4 paths, D = 1280 / 512 spline columns at 8 flops each): forward 8 D + 2 C T + C nW, layer-2 backward
# 6 C T + 8 D, layer-1 backward 4 C 16 + 8 D.
FLOPS_PER_EDGE = {"edge_l1_fwd": 8 * 512 + 2 * 128 * 16 + 128 * 4,
                  "edge_l1_bwd": 4 * 128 * 16 + 8 * 512,
                  "edge_l2_fwd": 8 * 1280 + 2 * 128 * 86 + 128 * 10,
                  "edge_l2_bwd": 6 * 128 * 86 + 8 * 1280}
# the density-projection layer 1 (64 hidden features per edge instead of 4 C weights): forward 8 H + 2 H 16,
# backward 8 H + 4 H 16, H = 64
FLOPS_PER_EDGE_L1D = {"edge_l1_fwd": 8 * 64 + 2 * 64 * 16, "edge_l1_bwd": 8 * 64 + 4 * 64 * 16}
# edge-kernel launches per evaluation: pass A l1_fwd, pass B l2_fwd + l2_bwd, pass C l1_bwd (pass C reads pass A's
# layer-1 results from the x1 cache, which the engine keeps whenever it fits)
# DRAM traffic of one launch of the dominant kernel: dram__bytes_read.sum + dram__bytes_write.sum of one
# 16,384-receiver k_edge_l2_bwd launch of the 24k-atom box (`ncu --set full --clock-control none -k regex:k_edge_l2_bwd
# -c 1 python bench.py --config water_24k --steps 1 --warmup 1 --no-e2e --no-cpu-baseline`), scaled per receiver to
# the 1.03M-atom box's 16,384-receiver chunks (same 84.6 edges per receiver).
TRAFFIC_PER_LAUNCH = {("water_24k", 16384, "edge_l2_bwd"): 560.42e6 + 82.16e6,
                      ("water_1m", 16384, "edge_l2_bwd"): 560.42e6 + 82.16e6}
EDGE_PASSES = {"edge_l1_fwd": 1, "edge_l1_bwd": 1, "edge_l2_fwd": 1, "edge_l2_bwd": 1}
ORDER = "lammps"      # atom order of the synthetic boxes (--order)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="water_1m", choices=list(CONFIGS))
    ap.add_argument("--chunk", type=int, default=16384)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-replica-check", action="store_true", help="multi-GPU: skip the single-GPU comparison")
    ap.add_argument("--md-steps", type=int, default=10, help="MD steps timed after the bench (0: none)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="multi-GPU: run the halo exchanges between whole passes instead of overlapping them with "
                         "interior chunks")
    ap.add_argument("--cpu-sample", type=int, default=8, help="water molecules per box edge of the CPU sample")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"])
    ap.add_argument("--skin", type=float, default=2.0, help="ghost shell = r_max + skin (multi-GPU)")
    ap.add_argument("--order", default="lammps", choices=["lammps", "morton", "grid"],
                    help="atom order: LAMMPS's spatial sort (bins of 3.5 A, x fastest), a Morton curve of 3 A cells "
                         "(the reference's standalone driver) or the generator's grid order")
    args = ap.parse_args()
    global ORDER
    ORDER = args.order
    if args.warmup < 1 or args.steps < 1:
        ap.error("--warmup and --steps must be >= 1 (the per-kernel breakdown is taken from the last warm-up step)")
    return args


def build_structure(cfg, grid=(1, 1, 1)):
    """The configuration's box; with grid != (1, 1, 1) its exact periodic replica (weak scaling): every rank's domain
    is then a copy of the single-GPU box, so each rank knows its atoms' energies and forces from one single-GPU
    evaluation (the reference's periodic-replica check, tests/gpu/test_threepass.py:80-87)."""
    from mace_onegpu import structures as S

    if cfg["kind"] == "water":
        cell = S.water_box(cfg["n"], seed=cfg["seed"])
    else:
        cell = S.alloy_bcc(cfg["n"], seed=cfg["seed"])
    if ORDER != "grid":
        o = S.morton_order(cell[0], cell[2]) if ORDER == "morton" else S.lammps_bin_order(cell[0], cell[2])
        cell = (cell[0][o], cell[1][o], cell[2])
    return cell if tuple(grid) == (1, 1, 1) else S.tile(*cell, grid)


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(self.idx)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ CPU baseline
CPU_CHUNK = 64      # the oracle's receiver chunk on the host: fastest there (chunk 16,384: 10x slower, page-fault bound)


def cpu_baseline(cfg, n_side: int):
    """The oracle (fp64 torch restatement of the three-pass evaluation, 512-knot tables) on a water box of
    n_side^3 molecules, all host threads, receiver chunks of CPU_CHUNK (the chunk changes only the size of the
    intermediates, not the arithmetic; 32-64 run fastest on the host, e.g. 78 against 7.5 atoms/s at 16,384 on a
    375-atom box with 8 cores).  Returns (atoms/s, seconds, cores, atoms)."""
    import dataclasses

    import torch

    from mace_onegpu import model as M
    from mace_onegpu import neighbors as NB
    from mace_onegpu import structures as S
    from oracle import mace_ref

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    m = M.default_model(cfg["model_seed"])
    if cfg["kind"] == "water":
        pos, Z, box = S.water_box(n_side, seed=cfg["seed"])
    else:
        pos, Z, box = S.alloy_bcc(max(n_side, 5), seed=cfg["seed"])
    cols = S.species_columns(Z, m.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(pos, box, m.arch.r_max)
    ref = mace_ref.MaceRef(m.params(), dataclasses.asdict(m.arch), spline_knots=512)
    t0 = time.perf_counter()
    ref.three_pass(pi, pj, rij, cols, len(Z), CPU_CHUNK)
    dt = time.perf_counter() - t0
    return len(Z) / dt, dt, cores, len(Z)


def run_reference(args, cfg, rank):
    if rank != 0:
        return
    vals = []
    for k in range(args.warmup + args.steps):
        v, dt, cores, n = cpu_baseline(cfg, args.cpu_sample)
        if k >= args.warmup:
            vals.append((v, dt))
    value = statistics.median(v for v, _ in vals)
    ms = statistics.median(dt for _, dt in vals) * 1e3
    sample = (f"oracle fp64 three-pass (512-knot tables, chunk {CPU_CHUNK}) on a {cfg['kind']} box of {n} atoms "
              f"({args.cpu_sample}^3 molecules) per step; atoms/s of this O(N) evaluation, which the per-atom cost "
              f"extrapolates linearly to the {cfg['desc'].split(':')[0]}")
    line = {"metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": {"workload": args.config, "description": cfg["desc"], "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ MD
def md_timing(args, cfg, m, eng, dev, world=1, rank=0, grid=(1, 1, 1)):
    """Velocity-Verlet MD on the bench's box (BASELINE config 3's schedule: dt 1 fs, Verlet skin 2 A,
    Maxwell-Boltzmann velocities at 300 K), timed over args.md_steps steps with CUDA events after the
    force-evaluation timing (max over ranks).  One GPU: mace_onegpu.md.VelocityVerlet.  N GPUs: DomainVelocityVerlet
    on the same domains as the force bench (replicated positions, each rank's domain forces with the halo
    exchanges, one force all-reduce per step, decomposition and Verlet lists rebuilt on the GPU).  The random-init
    model (energy scale 100) heats water within tens of fs, so this is a timing figure of the MD loop (force
    evaluation, Verlet-list filter / rebuild, integration), not physics."""
    import torch

    from mace_onegpu import structures as S
    from mace_onegpu.md import DomainVelocityVerlet, VelocityVerlet

    pos, Z, box = build_structure(cfg, grid if args.scaling == "weak" else (1, 1, 1))
    cols = S.species_columns(Z, m.arch.atomic_numbers)
    vel = S.maxwell_boltzmann(Z, 300.0, seed=0)
    if world == 1:
        md = VelocityVerlet(eng, pos, box, cols, Z, vel, dt=1.0, skin=args.skin)
    else:
        import torch.distributed as dist

        md = DomainVelocityVerlet(eng, pos, box, cols, Z, vel, grid, rank, dt=1.0, skin=args.skin,
                                  overlap=not args.no_overlap)
    md.step()                                           # warm-up step
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0.record()
    for _ in range(args.md_steps):
        md.step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    sps = args.md_steps / (ms * 1e-3)
    out = {"md_ns_per_day": sps * 1.0 * 86400 / 1e6, "steps_per_s": sps, "steps": args.md_steps, "dt_fs": 1.0,
           "skin_A": args.skin, "atoms": len(Z), "neighbour_rebuilds": md.rebuilds,
           "driver": "VelocityVerlet" if world == 1 else "DomainVelocityVerlet (replicated positions, domain forces, "
                                                         "one force all-reduce per step)",
           "note": "random-init model: a timing figure of the MD loop, not a physical trajectory"}
    del md
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------------ replica check
def replica_check(args, cfg, m, dev, eng, step, hx, gid, n, nt, pi, pj, n_cell):
    """Multi-GPU correctness inside every scaling run.  Each rank evaluates the single-GPU box (the weak-scaling
    cell, or the whole box under strong scaling) on its own GPU, then compares its domain's last distributed
    evaluation atom by atom: energy of every local atom against its image's, atom force (ghost contributions
    returned to their owners by a reverse halo exchange) against its image's, and the total energy against N times
    (weak) or once (strong) the single-GPU total.  Collective steps are the same on every rank."""
    import torch
    import torch.distributed as dist

    from mace_onegpu import neighbors as NB
    from mace_onegpu import structures as S
    from mace_onegpu.engine import ThreePassEngine

    eat, pf = step()
    eat = eat.clone()
    F = torch.zeros(nt, 3, dtype=torch.float32, device=dev)
    F.index_add_(0, pi.long(), (-pf).float())
    F.index_add_(0, pj.long(), pf.float())
    hx.reverse(F)
    cpos, cZ, cbox = build_structure(cfg)
    ccols = torch.as_tensor(S.species_columns(cZ, m.arch.atomic_numbers))
    rpi, rpj, rrij = NB.neighbor_list(cpos, cbox, m.arch.r_max, device=dev)
    reng = ThreePassEngine(m, sorted(set(ccols.tolist())), chunk=args.chunk, device=dev)
    reat, rpf = reng.evaluate(reng.plan(rpi, rpj, rrij, ccols.to(dev), n_cell, n_cell))
    rF = torch.zeros(n_cell, 3, dtype=torch.float64, device=dev)
    rF.index_add_(0, rpi.long(), -rpf)
    rF.index_add_(0, rpj.long(), rpf)
    img = torch.as_tensor(gid[:n] % n_cell, device=dev)
    stats = torch.tensor([(eat - reat[img]).abs().max().item(), (F[:n].double() - rF[img]).abs().max().item()],
                         dtype=torch.float64, device=dev)
    esum = torch.tensor([eat.sum().item()], dtype=torch.float64, device=dev)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    dist.all_reduce(esum)
    copies = dist.get_world_size() if args.scaling == "weak" else 1
    e1 = float(reat.sum().item())
    del reng
    torch.cuda.empty_cache()
    return {"max_dE_eV": stats[0].item(), "max_dF_eV_per_A": stats[1].item(), "E_total_eV": esum.item(),
            "E_single_gpu_x_copies_eV": copies * e1, "rel_dE_total": abs(esum.item() - copies * e1) / abs(copies * e1),
            "tolerance": {"dE_eV": 1e-5, "dF_eV_per_A": 1e-3},
            "ok": bool(stats[0].item() < 1e-5 and stats[1].item() < 1e-3),
            "reference": f"single-GPU evaluation of the {n_cell}-atom periodic box on every rank"}


# ------------------------------------------------------------------------------------------------ B200 arm
def main():
    args = parse()
    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa = False
    if world > 1:
        import datetime

        from mace_onegpu import hostio

        numa = hostio.bind_to_gpu_numa(dev)    # pinned e2e buffers on the GPU's NUMA node (first touch)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from mace_onegpu import _native as N
    from mace_onegpu import model as M
    from mace_onegpu import neighbors as NB
    from mace_onegpu import structures as S
    from mace_onegpu.engine import ThreePassEngine
    from mace_onegpu.mliap_data import MLIAPData
    from mace_onegpu.mliap_threepass import ThreePassMLIAP

    m = M.default_model(cfg["model_seed"])
    hx = None
    if world == 1:
        pos, Z, box = build_structure(cfg)
        cols_all = torch.as_tensor(S.species_columns(Z, m.arch.atomic_numbers))
        pi, pj, rij = NB.neighbor_list(pos, box, m.arch.r_max, device=dev)
        n = nt = len(Z)
        cols = cols_all
        parallelism = "single"
    else:
        from mace_onegpu import domain as DM

        grid = DM.grid_for(world)
        pos, Z, box = build_structure(cfg, grid if args.scaling == "weak" else (1, 1, 1))
        n_cell = len(Z) // (world if args.scaling == "weak" else 1)
        cols_all = torch.as_tensor(S.species_columns(Z, m.arch.atomic_numbers))
        dec = DM.DeviceDecomposition(torch.as_tensor(pos, device=dev), box, grid, m.arch.r_max + args.skin)
        p, gid, n = dec.rank_atoms(rank)
        nt = int(gid.numel())
        pi, pj, rij = NB.neighbor_list_open(p, n, m.arch.r_max, device=dev)
        cols = cols_all[gid.cpu()]
        hx = DM.HaloExchange(dec, rank, dev)
        del dec, p
        parallelism = (f"domain {grid[0]}x{grid[1]}x{grid[2]}, NCCL halo exchange "
                       f"({'between passes' if args.no_overlap else 'overlapped with interior chunks'}), "
                       f"ghost shell {m.arch.r_max + args.skin:g} A, {hx.n_interior} interior atoms on rank 0")
    P = int(pi.numel())
    elems = cols.to(dev)
    eng = ThreePassEngine(m, sorted(set(cols_all.tolist())), chunk=args.chunk, device=dev)
    n_all = torch.tensor([n], device=dev, dtype=torch.int64)
    if world > 1:
        dist.all_reduce(n_all)
    n_total = int(n_all.item())

    def step():
        plan = eng.plan(pi, pj, rij, elems, n, nt)
        if hx is None:
            return eng.evaluate(plan)
        if args.no_overlap:
            return eng.evaluate(plan, hx.forward, hx.reverse)
        return eng.evaluate(plan, halo=hx)

    # the per-kind breakdown comes from the last warm-up step; inside the timed region only the roofline kernel is
    # recorded (every recorded launch adds two event records to the stream: all kinds cost ~1% of the step time)
    fpe = dict(FLOPS_PER_EDGE, **(FLOPS_PER_EDGE_L1D if eng.fm.l1_density else {}))
    N.timing_kinds(None)
    for w in range(args.warmup):
        if w == args.warmup - 1:
            N.timing(True)
        step()
    torch.cuda.synchronize()
    warm = N.timing(False)
    dom = max((k for k in warm if k in fpe), key=lambda k: warm[k][0])
    N.timing_kinds([dom])
    barrier()
    clk = ClockSampler(local)
    clk.start()
    N.timing(True)
    launches0 = N.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    barrier()
    launches = N.launch_count() - launches0
    kern = N.timing(False)
    N.timing_kinds(None)
    clocks = clk.stop()
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_per_step = ms / args.steps
    value = n_total * args.steps / (ms * 1e-3)

    # roofline of the dominant kernel (FP32 SIMT edge kernels: FLOP/s against the measured FFMA issue ceiling)
    dom_ms, dom_launches = kern[dom]
    flops = fpe[dom] * P * EDGE_PASSES[dom] * args.steps
    achieved = flops / (dom_ms * 1e-3) / 1e12 if dom_ms > 0 else 0.0
    scratch = torch.zeros(1, device=dev)
    pk = N.c_f64()
    N.check(N.lib().mace_b200_ffma_peak(2000, N.ptr(scratch), N.byref(pk), torch.cuda.current_stream().cuda_stream),
            "ffma_peak")
    peak = pk.value

    # e2e through the reference-facing ML-IAP call, host buffers, copies in the timed region
    e2e = None
    if not args.no_e2e:
        mli = ThreePassMLIAP(m, chunk=args.chunk)
        hpi = pi.cpu().pin_memory()
        hpj = pj.cpu().pin_memory()
        hrij = rij.cpu().pin_memory()
        hel = cols.clone().pin_memory()
        data = MLIAPData(hpi, hpj, hrij, hel, n, host_outputs=True, exchange=hx)
        for _ in range(max(1, args.warmup)):
            mli.compute_forces(data)
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            mli.compute_forces(data)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ems = e0.elapsed_time(e1)
        if world > 1:
            tt = torch.tensor([ems], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ems = float(tt.item())
        e2e = {"value": n_total * args.steps / (ems * 1e-3), "unit": "atoms/s",
               "h2d_bytes_per_step": int(P * (4 + 4 + 24) + nt * 8), "d2h_bytes_per_step": int(n * 8 + P * 24)}
        # one more call with CUDA events between the passes and around the streamed pair-list copies (not timed)
        mli._eng.pass_timing = True
        mli.compute_forces(data)
        e2e["breakdown_s"] = {k: round(v, 5) for k, v in mli._eng.pass_times().items()}
        mli._eng.pass_timing = False

    md = None
    if args.md_steps > 0:
        md = md_timing(args, cfg, m, eng, dev, world, rank, grid if world > 1 else (1, 1, 1))

    replica = None
    if world > 1 and not args.no_replica_check:
        replica = replica_check(args, cfg, m, dev, eng, step, hx, gid, n, nt, pi, pj, n_cell)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, dt, cores, na = cpu_baseline(cfg, args.cpu_sample)
        cpu = {"value": v, "unit": "atoms/s", "cores": cores, "kind": "port",
               "sample": f"oracle fp64 three-pass (512-knot tables, chunk {CPU_CHUNK}) on a {na}-atom {cfg['kind']} box "
                         f"({args.cpu_sample}^3 molecules), {dt:.1f} s; atoms/s of this O(N) evaluation, "
                         f"extrapolated linearly per atom to the workload"}

    if rank == 0:
        kinds = {k: {"ms_per_step": v[0], "launches_per_step": v[1], "source": "last warm-up step"}
                 for k, v in warm.items()}
        kinds[dom] = {"ms_per_step": dom_ms / args.steps, "launches_per_step": dom_launches / args.steps,
                      "source": "timed region"}
        line = {"metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": args.scaling if world > 1 else "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": args.config, "description": cfg["desc"], "atoms_total": n_total,
                           "atoms_rank0": n, "ghosts_rank0": nt - n, "pairs_rank0": P, "chunk": args.chunk,
                           "spline_knots": 512, "model": "MACE-MPA-0-medium architecture, random init",
                           "parallelism": parallelism, "gemm": "tcgen05 3xTF32" if eng.fm.use_tc else "SIMT fp32",
                           "layer1": "density projection" if eng.fm.l1_density else "direct",
                           "host_numa_bound": numa,
                           "l2": "inputs larger than L2 (no flush)", "atom_order": ORDER,
                           "peak_device_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 2)},
                "roofline": {"bound": "fp32", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak,
                             "traffic": TRAFFIC_PER_LAUNCH.get((args.config, args.chunk, dom)),
                             "traffic_unit": "bytes per launch (ncu dram__bytes_read + dram__bytes_write)",
                             "traffic_source": "one-launch capture on the 24k-atom box (16,384 receivers), scaled per "
                                               "receiver (profiles/k_edge_l2_bwd_water24k.md)",
                             "peak_source": "FFMA issue ceiling measured in this run (mace_b200_ffma_peak)",
                             "flops_per_edge": fpe[dom]},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks, "kernels": kinds,
                "replica_check": replica, "md": md}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
