"""Spatial domain decomposition and the distributed H1 / G1 halo exchanges, on CPU: ghost completeness against the
minimum-image pair list, and a 2-rank gloo run of the oracle's three-pass evaluation reproducing the single-process
energies and forces (the multi-GPU path's host logic; the GPU run uses the same classes over NCCL)."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mace_onegpu import domain as D
from mace_onegpu import model as M
from mace_onegpu import neighbors as NB
from mace_onegpu import structures as S


def _pairs_set(pi, pj, rij):
    return {(int(a), int(b), tuple(np.round(r, 8))) for a, b, r in zip(pi, pj, rij)}


@pytest.mark.parametrize("grid", [(2, 1, 1), (1, 2, 2), (2, 2, 2)])
def test_ghosts_reproduce_minimum_image_pairs(grid):
    pos, Z, box = S.water_box(5, seed=3)
    r = 6.0
    pi, pj, rij = NB.neighbor_list(pos, box, r)
    ref = _pairs_set(pi.numpy(), pj.numpy(), rij.numpy())
    dec = D.Decomposition(pos, box, grid, r)
    got = set()
    for rank in range(dec.nranks):
        p, gid, nl = dec.rank_atoms(rank)
        qi, qj, qr = NB.neighbor_list_open(p, nl, r)
        got |= _pairs_set(gid[qi.numpy()], gid[qj.numpy()], qr.numpy())
        # receive blocks are contiguous and match the owners' send lists
        blocks = dec.recv_blocks(rank)
        for o, (g0, g1) in blocks.items():
            assert np.array_equal(dec.local[o][dec.send_list(o, rank)], gid[nl + g0:nl + g1])
    assert got == ref


@pytest.mark.parametrize("grid,r_ghost", [((2, 1, 1), 8.0), ((1, 2, 1), 8.0), ((2, 2, 1), 8.0), ((2, 2, 2), 8.0),
                                          ((3, 1, 1), 8.0), ((4, 2, 1), 7.5), ((1, 1, 1), 8.0)])
def test_device_decomposition_equals_numpy(grid, r_ghost):
    """DeviceDecomposition (torch, used on the GPU by the multi-GPU bench and MD) builds exactly the numpy
    construction: owners, local order, ghost sets and ghost order, exchange maps, rank positions."""
    pos, Z, box = S.water_box(10, 9, 8, seed=5)
    a = D.Decomposition(pos, box, grid, r_ghost)
    b = D.DeviceDecomposition(torch.as_tensor(pos), box, grid, r_ghost)
    assert np.array_equal(a.owner, b.owner.numpy())
    for r in range(a.nranks):
        assert np.array_equal(a.local[r], b.local[r].numpy())
        assert np.array_equal(a.ghost[r], b.ghost[r].numpy())
        assert a.n_interior[r] == b.n_interior[r] and a.recv_blocks(r) == b.recv_blocks(r)
        for p in range(a.nranks):
            assert np.array_equal(a.send_list(r, p), b.send_list(r, p).numpy())
        pa, ga, na = a.rank_atoms(r)
        pb, gb, nb = b.rank_atoms(r)
        assert na == nb and np.array_equal(ga, gb.numpy()) and np.array_equal(pa, pb.numpy())


@pytest.mark.parametrize("grid", [(2, 1, 1), (1, 2, 1)])
def test_interior_atoms_first_have_no_ghost_neighbours(grid):
    """Each rank's local atoms are ordered interior first: receivers [0, n_interior) have only local senders and are
    in no rank's ghost list, so their chunks may run while a halo exchange is in flight (engine._run_overlap).  The
    box leaves every domain wider than twice the 8 A ghost shell, so that it has interior atoms."""
    pos, Z, box = S.water_box(*((14, 8, 8) if grid[0] == 2 else (8, 14, 8)), seed=1)
    r = 6.0
    dec = D.Decomposition(pos, box, grid, r + 2.0)
    ghosts_of = {int(a) for g in dec.ghost for a in g[:, 0]}
    for rank in range(dec.nranks):
        p, gid, nl = dec.rank_atoms(rank)
        ni = dec.n_interior[rank]
        assert 0 < ni < nl
        assert not ({int(a) for a in gid[:ni]} & ghosts_of)
        assert {int(a) for a in gid[ni:nl]} <= ghosts_of
        qi, qj, _ = NB.neighbor_list_open(p, nl, r)
        inner = qi < ni
        assert bool((qj[inner] < nl).all())


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, grid, out_q):
    import torch.distributed as dist

    from oracle import mace_ref

    torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        mdl = M.default_model(0)
        pos, Z, box = S.water_box(4, seed=0)
        cols = S.species_columns(Z, mdl.arch.atomic_numbers)
        dec = D.Decomposition(pos, box, grid, mdl.arch.r_max)
        p, gid, nl = dec.rank_atoms(rank)
        pi, pj, rij = NB.neighbor_list_open(p, nl, mdl.arch.r_max)
        hx = D.HaloExchange(dec, rank, "cpu")
        ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch))
        eat, pf = ref.three_pass(pi, pj, rij, cols[gid], nl, 64, forward_exchange=hx.forward,
                                 reverse_exchange=hx.reverse)
        n = len(Z)
        E = torch.zeros(n, dtype=torch.float64)
        E[torch.as_tensor(gid[:nl])] = eat
        F = torch.zeros(n, 3, dtype=torch.float64)
        F.index_add_(0, torch.as_tensor(gid[pi.numpy()]), -pf)
        F.index_add_(0, torch.as_tensor(gid[pj.numpy()]), pf)
        dist.all_reduce(E)
        dist.all_reduce(F)
        if rank == 0:
            out_q.put((E.numpy(), F.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("grid", [(2, 1, 1)])
def test_two_rank_gloo_three_pass_matches_single_process(grid):
    from oracle import mace_ref

    world = int(np.prod(grid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, grid, q)) for r in range(world)]
    for p_ in procs:
        p_.start()
    import queue
    import time

    t0 = time.time()
    while True:
        try:
            E, F = q.get(timeout=2)
            break
        except queue.Empty:
            dead = [p_.exitcode for p_ in procs if p_.exitcode not in (None, 0)]
            assert not dead and time.time() - t0 < 600, f"worker failed: exit codes {dead}"
    for p_ in procs:
        p_.join(timeout=120)
        assert p_.exitcode == 0
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(4, seed=0)
    cols = S.species_columns(Z, mdl.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch))
    e0, pf0 = ref.three_pass(pi, pj, rij, cols, len(Z), 64)
    F0 = mace_ref.atom_forces(pi, pj, pf0, len(Z)).numpy()
    assert np.abs(E - e0.numpy()).max() < 1e-9
    assert np.abs(F - F0).max() < 1e-9


def test_device_decomposition_atoms_on_domain_faces():
    """Atoms exactly on domain faces, at the box origin and one ulp below the box length: both constructions put
    them in the same domains and ghost sets."""
    pos, Z, box = S.water_box(10, 9, 8, seed=6)
    w = box / np.array([2, 2, 2])
    pos = pos.copy()
    pos[0] = [w[0], w[1], w[2]]                          # on three faces at once
    pos[1] = [0.0, 0.0, 0.0]
    pos[2] = np.nextafter(box, 0.0)                       # just inside the upper box faces
    pos[3] = [w[0] - 8.0, w[1] + 8.0, 0.5 * w[2]]          # exactly one ghost shell from a face
    a = D.Decomposition(pos, box, (2, 2, 2), 8.0)
    b = D.DeviceDecomposition(torch.as_tensor(pos), box, (2, 2, 2), 8.0)
    assert np.array_equal(a.owner, b.owner.numpy())
    for r in range(a.nranks):
        assert np.array_equal(a.local[r], b.local[r].numpy())
        assert np.array_equal(a.ghost[r], b.ghost[r].numpy())
