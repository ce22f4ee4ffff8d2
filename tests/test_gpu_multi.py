"""Multi-GPU parity: the three-pass evaluation split over 2 GPUs by spatial domains (explicit ghosts, H1 forward /
G1 reverse halo exchange over NCCL, between whole passes or overlapped with interior chunks on a side stream)
reproduces the single-process fp64 oracle.  Needs >= 2 GPUs (skipped otherwise);
ranks run as child processes; NVLS is off (NCCL_NVLS_ENABLE=0) and the process group has a short timeout."""
import dataclasses
import functools
import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mace_onegpu import domain as D
from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import structures as S

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, grid, out_q, overlap):
    import datetime

    import torch.distributed as dist

    from mace_onegpu.engine import ThreePassEngine

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        mdl = M.default_model(0)
        pos, Z, box = S.water_box(16, 8, 8, seed=2)
        cols = S.species_columns(Z, mdl.arch.atomic_numbers)
        dec = D.Decomposition(pos, box, grid, mdl.arch.r_max + 2.0)
        p, gid, nl = dec.rank_atoms(rank)
        pi, pj, rij = NB.neighbor_list_open(p, nl, mdl.arch.r_max, device=dev)
        eng = ThreePassEngine(mdl, sorted(set(cols.tolist())), chunk=32, device=dev)
        hx = D.HaloExchange(dec, rank, dev)
        plan = eng.plan(pi, pj, rij, torch.as_tensor(cols[gid]), nl, len(gid))
        if overlap:
            assert hx.n_interior >= 32                   # at least one interior chunk runs under each exchange
            eat, pf = eng.evaluate(plan, halo=hx)
        else:
            eat, pf = eng.evaluate(plan, hx.forward, hx.reverse)
        torch.cuda.synchronize()
        n = len(Z)
        E = torch.zeros(n, dtype=torch.float64, device=dev)
        E[torch.as_tensor(gid[:nl], device=dev)] = eat
        F = torch.zeros(n, 3, dtype=torch.float64, device=dev)
        gi = torch.as_tensor(gid, device=dev)
        F.index_add_(0, gi[pi.long()], -pf)
        F.index_add_(0, gi[pj.long()], pf)
        dist.all_reduce(E)
        dist.all_reduce(F)
        if rank == 0:
            out_q.put((E.cpu().numpy(), F.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@functools.lru_cache(maxsize=1)
def _oracle():
    from oracle import mace_ref

    mdl = M.default_model(0)
    pos, Z, box = S.water_box(16, 8, 8, seed=2)
    cols = S.species_columns(Z, mdl.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), spline_knots=512)
    e0, pf0 = ref.three_pass(pi, pj, rij, cols, len(Z), 512)
    return e0, mace_ref.atom_forces(pi, pj, pf0, len(Z)).numpy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("overlap", [False, True], ids=["between-passes", "overlapped"])
def test_two_gpu_domain_decomposition_matches_oracle(overlap):

    grid, world = (2, 1, 1), 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, grid, q, overlap)) for r in range(world)]
    for p_ in procs:
        p_.start()
    t0 = time.time()
    while True:
        try:
            E, F = q.get(timeout=2)
            break
        except queue.Empty:
            dead = [p_.exitcode for p_ in procs if p_.exitcode not in (None, 0)]
            assert not dead and time.time() - t0 < 600, f"rank failed: exit codes {dead}"
    for p_ in procs:
        p_.join(timeout=120)
        assert p_.exitcode == 0
    e0, F0 = _oracle()
    assert np.abs(E - e0.numpy()).max() < 1e-5
    assert np.abs(F - F0).max() < 1e-3


MD_STEPS = 8
MD_REBUILD_AT = 4      # one forced rebuild (wraps positions, new domains and lists) besides the automatic ones


def _md_worker(rank, world, port, out_q):
    """DomainVelocityVerlet over 2 GPUs; rank 0 then runs the single-GPU VelocityVerlet on the same box."""
    import datetime

    import torch.distributed as dist

    from mace_onegpu.engine import ThreePassEngine
    from mace_onegpu.md import DomainVelocityVerlet, VelocityVerlet

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        mdl = M.default_model(0)
        pos, Z, box = S.water_box(16, 8, 8, seed=2)
        cols = S.species_columns(Z, mdl.arch.atomic_numbers)
        vel = S.maxwell_boltzmann(Z, 300.0, seed=0)
        eng = ThreePassEngine(mdl, sorted(set(cols.tolist())), chunk=256, device=dev)
        md = DomainVelocityVerlet(eng, pos, box, cols, Z, vel, (2, 1, 1), rank, dt=1.0, skin=1.0)
        E = [md.epot]
        for k in range(MD_STEPS):
            if k == MD_REBUILD_AT:
                md._build()
            md.step()
            E.append(md.epot)
        torch.cuda.synchronize()
        x2, v2 = md.x.cpu().numpy(), md.v.cpu().numpy()
        xs = [torch.zeros_like(md.x) for _ in range(world)]
        dist.all_gather(xs, md.x)
        same = all(torch.equal(xs[0], t) for t in xs)
        nb2 = md.rebuilds
        del md
        dist.barrier()
        if rank == 0:
            one = VelocityVerlet(eng, pos, box, cols, Z, vel, dt=1.0, skin=1.0)
            E1 = [one.epot]
            for k in range(MD_STEPS):
                if k == MD_REBUILD_AT:
                    one._build()
                one.step()
                E1.append(one.epot)
            out_q.put((x2, v2, np.array(E), nb2, same, one.x.cpu().numpy(), one.v.cpu().numpy(), np.array(E1),
                       one.rebuilds, len(Z), np.asarray(box)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_md_matches_single_gpu_md():
    """Eight velocity-Verlet steps (dt 1 fs, skin 1 A; the decomposition and Verlet lists are rebuilt on the GPU at
    least once along the way) over 2 GPUs follow the single-GPU trajectory to within the fp32 force noise, and the
    replicated positions stay identical on both ranks.  Positions are compared under minimum image: a rebuild wraps
    them into the box."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_md_worker, args=(r, 2, port, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    t0 = time.time()
    while True:
        try:
            res = q.get(timeout=2)
            break
        except queue.Empty:
            dead = [p_.exitcode for p_ in procs if p_.exitcode not in (None, 0)]
            assert not dead and time.time() - t0 < 600, f"rank failed: exit codes {dead}"
    for p_ in procs:
        p_.join(timeout=120)
        assert p_.exitcode == 0
    x2, v2, E2, nb2, same, x1, v1, E1, nb1, n, box = res
    assert same
    assert nb2 == nb1 >= 2
    d = x2 - x1
    d -= box * np.round(d / box)
    assert np.abs(d).max() < 1e-5
    assert np.abs(v2 - v1).max() < 1e-5
    assert np.abs(E2 - E1).max() < 1e-5 * n
