"""Full neighbour list (both directions) of an orthorhombic periodic box: cell list + minimum image, in torch so that
it runs on the host or on the GPU (input preparation for the standalone driver; the force evaluation itself takes the
pair list as given, like the ML-IAP boundary).  The algorithm is the one of the reference's
``System.build_neighbors`` (``mace_onegpu/receiver_chunk_mace.py:114-165``): 27-cell candidates per atom, a count
pass then a fill pass, brute force when a box dimension holds fewer than 3 cells.

Output convention: pairs sorted by receiver i, rij = x_i - x_j (minimum image), the edge vector of mace's
``get_edge_vectors_and_lengths`` (receiver minus sender).  On a CUDA device (and at least 3 cells per periodic
dimension) the lists come from the library's cell-list kernels (mace_b200_nbr_count / _fill, one warp per receiver,
senders of a receiver in a fixed cell-scan order); on the host the torch version below sorts senders by index.
``verlet_filter`` reduces a skin list to the pairs within the cutoff at new positions (mace_b200_verlet_filter).
"""
from __future__ import annotations

import ctypes

import torch


def _cells(pos, lo, width, nc):
    """cell_start int32 [ncell + 1], cell_atoms int32 [n] (atoms grouped by cell, ascending index within a cell) with
    the kernels' cell formula clamp(floor((x - lo) * (1 / width)))."""
    c = torch.floor((pos - lo) * (1.0 / width)).long()
    c = torch.minimum(torch.clamp(c, min=0), nc - 1)
    lin = (c[:, 0] * nc[1] + c[:, 1]) * nc[2] + c[:, 2]
    order = torch.argsort(lin, stable=True)
    ncell = int(nc.prod())
    start = torch.zeros(ncell + 1, dtype=torch.int32, device=pos.device)
    start[1:] = torch.cumsum(torch.bincount(lin, minlength=ncell), 0).to(torch.int32)
    return start, order.to(torch.int32).contiguous()


def _d3(v):
    return (ctypes.c_double * 3)(*[float(x) for x in v])


def _cuda_pairs(pos, n_recv: int, lo, width, nc, box, periodic: bool, r_cut: float, return_rowptr: bool = False):
    from . import _native as N

    L = N.lib()
    st = torch.cuda.current_stream(pos.device).cuda_stream
    start, atoms = _cells(pos, lo, width, nc)
    lo_a, w_a, box_a = _d3(lo.tolist()), _d3(width.tolist()), _d3(box.tolist() if periodic else [0.0] * 3)
    nc_a = (ctypes.c_int32 * 3)(*[int(x) for x in nc.tolist()])
    grid = (ctypes.addressof(lo_a), ctypes.addressof(w_a), ctypes.addressof(nc_a), ctypes.addressof(box_a))
    counts = torch.empty(n_recv, dtype=torch.int32, device=pos.device)
    N.check(L.mace_b200_nbr_count(N.ptr(pos), N.ptr(start), N.ptr(atoms), *grid, int(periodic), n_recv, float(r_cut),
                                  N.ptr(counts), st), "nbr_count")
    rowptr = torch.zeros(n_recv + 1, dtype=torch.int64, device=pos.device)
    rowptr[1:] = torch.cumsum(counts, 0)
    P = int(rowptr[-1].item())
    pi = torch.empty(P, dtype=torch.int32, device=pos.device)
    pj = torch.empty(P, dtype=torch.int32, device=pos.device)
    rij = torch.empty(P, 3, dtype=torch.float64, device=pos.device)
    status = torch.zeros(1, dtype=torch.int32, device=pos.device)
    N.check(L.mace_b200_nbr_fill(N.ptr(pos), N.ptr(start), N.ptr(atoms), *grid, int(periodic), n_recv, float(r_cut),
                                 N.ptr(rowptr), N.ptr(pi), N.ptr(pj), N.ptr(rij), N.ptr(status), st), "nbr_fill")
    if int(status.item()):
        raise RuntimeError("nbr_fill: pair count changed between the count and fill passes")
    return (pi, pj, rij, rowptr) if return_rowptr else (pi, pj, rij)


def verlet_filter(pos, box, vrow, vj, r_cut: float):
    """Pairs of the skin list (CSR vrow int64 [n + 1], vj int32) within r_cut at positions `pos` (CUDA, periodic
    minimum image in `box`): (pi int32, pj int32, rij fp64 [P, 3]) in the skin list's order."""
    from . import _native as N

    L = N.lib()
    st = torch.cuda.current_stream(pos.device).cuda_stream
    n = vrow.numel() - 1
    box_a = _d3(torch.as_tensor(box).tolist())
    counts = torch.empty(n, dtype=torch.int32, device=pos.device)
    N.check(L.mace_b200_verlet_filter(N.ptr(pos), ctypes.addressof(box_a), 1, n, N.ptr(vrow), N.ptr(vj),
                                      float(r_cut), N.ptr(counts), None, None, None, None, None, st), "verlet_filter")
    rowptr = torch.zeros(n + 1, dtype=torch.int64, device=pos.device)
    rowptr[1:] = torch.cumsum(counts, 0)
    P = int(rowptr[-1].item())
    pi = torch.empty(P, dtype=torch.int32, device=pos.device)
    pj = torch.empty(P, dtype=torch.int32, device=pos.device)
    rij = torch.empty(P, 3, dtype=torch.float64, device=pos.device)
    status = torch.zeros(1, dtype=torch.int32, device=pos.device)
    N.check(L.mace_b200_verlet_filter(N.ptr(pos), ctypes.addressof(box_a), 1, n, N.ptr(vrow), N.ptr(vj),
                                      float(r_cut), None, N.ptr(rowptr), N.ptr(pi), N.ptr(pj), N.ptr(rij),
                                      N.ptr(status), st), "verlet_filter")
    if int(status.item()):
        raise RuntimeError("verlet_filter: pair count changed between the count and fill passes")
    return pi, pj, rij


def neighbor_list(pos, box, r_max: float, device="cpu", block: int = 16384, return_rowptr: bool = False):
    """Returns (pi int32 [P], pj int32 [P], rij float64 [P, 3]) for all 0 < |x_i - x_j|_mic < r_max (and the receiver
    row pointer int64 [N + 1] with return_rowptr)."""
    pos = torch.as_tensor(pos, dtype=torch.float64, device=device)
    box = torch.as_tensor(box, dtype=torch.float64, device=device)
    if not bool((box > 2.0 * r_max).all()):
        raise ValueError("minimum image needs every box length > 2 r_max")
    pos = torch.remainder(pos, box).contiguous()
    N = pos.shape[0]
    r2 = r_max * r_max
    nc = torch.clamp((box / r_max).floor().long(), min=1)
    brute = bool((nc < 3).any())
    if pos.is_cuda and not brute:
        zero = torch.zeros(3, dtype=torch.float64, device=pos.device)
        return _cuda_pairs(pos, N, zero, box / nc, nc, box, True, r_max, return_rowptr)
    if not brute:
        c = torch.minimum((pos / (box / nc)).floor().long(), nc - 1)
        lin = (c[:, 0] * nc[1] + c[:, 1]) * nc[2] + c[:, 2]
        order = torch.argsort(lin, stable=True)
        lin_sorted = lin[order]
        ncell = int(nc.prod())
        counts = torch.bincount(lin_sorted, minlength=ncell)
        start = torch.cumsum(counts, 0) - counts
        mcc = int(counts.max())
        offs = torch.stack(torch.meshgrid(*[torch.arange(-1, 2, device=device)] * 3, indexing="ij"), -1).reshape(27, 3)
    out_i, out_j = [], []
    for a in range(0, N, block):
        b = min(a + block, N)
        ri = torch.arange(a, b, device=device)
        if brute:
            cand = torch.arange(N, device=device).unsqueeze(0).expand(b - a, N)
            valid = torch.ones_like(cand, dtype=torch.bool)
        else:
            cc = (c[a:b].unsqueeze(1) + offs.unsqueeze(0)) % nc
            cl = (cc[..., 0] * nc[1] + cc[..., 1]) * nc[2] + cc[..., 2]
            k = torch.arange(mcc, device=device)
            slot = start[cl].unsqueeze(-1) + k
            valid = (k < counts[cl].unsqueeze(-1)).reshape(b - a, -1)
            cand = order[torch.where(valid, slot.reshape(b - a, -1), torch.zeros_like(valid, dtype=torch.long))]
        d = pos[ri].unsqueeze(1) - pos[cand]
        d = d - box * torch.round(d / box)
        ok = valid & ((d * d).sum(-1) < r2) & (cand != ri.unsqueeze(1))
        ii, kk = ok.nonzero(as_tuple=True)
        out_i.append(ii + a)
        out_j.append(cand[ii, kk])
    pi = torch.cat(out_i)
    pj = torch.cat(out_j)
    key = pi * N + pj
    o = torch.argsort(key)
    pi, pj = pi[o], pj[o]
    rij = pos[pi] - pos[pj]
    rij = rij - box * torch.round(rij / box)
    if return_rowptr:
        rowptr = torch.searchsorted(pi, torch.arange(N + 1, device=pi.device))
        return pi.to(torch.int32), pj.to(torch.int32), rij, rowptr
    return pi.to(torch.int32), pj.to(torch.int32), rij


def neighbor_list_open(pos, n_recv: int, r_max: float, device="cpu", block: int = 16384):
    """Pairs of an open (non-periodic) point set with explicit ghost images: receivers are atoms [0, n_recv),
    senders any atom, 0 < |x_i - x_j| < r_max.  Cell list over the bounding box (cells >= r_max, 27 neighbours
    without wrap).  Returns (pi int32, pj int32, rij fp64 = x_i - x_j) sorted by (pi, pj)."""
    pos = torch.as_tensor(pos, dtype=torch.float64, device=device).contiguous()
    N = pos.shape[0]
    lo = pos.min(0).values
    ext = pos.max(0).values - lo
    nc = torch.clamp((ext / r_max).floor().long(), min=1)
    if pos.is_cuda:
        width = torch.maximum(ext / nc, torch.full_like(ext, r_max))
        return _cuda_pairs(pos, n_recv, lo, width, nc, lo, False, r_max)
    c = torch.minimum(((pos - lo) / (ext / nc + 1e-12)).floor().long(), nc - 1)
    lin = (c[:, 0] * nc[1] + c[:, 1]) * nc[2] + c[:, 2]
    order = torch.argsort(lin, stable=True)
    ncell = int(nc.prod())
    counts = torch.bincount(lin, minlength=ncell)
    start = torch.cumsum(counts, 0) - counts
    mcc = int(counts.max())
    offs = torch.stack(torch.meshgrid(*[torch.arange(-1, 2, device=device)] * 3, indexing="ij"), -1).reshape(27, 3)
    r2 = r_max * r_max
    out_i, out_j = [], []
    for a in range(0, n_recv, block):
        b = min(a + block, n_recv)
        ri = torch.arange(a, b, device=device)
        cc = c[a:b].unsqueeze(1) + offs.unsqueeze(0)                          # [n, 27, 3]
        inb = ((cc >= 0) & (cc < nc)).all(-1)
        cc = torch.where(inb.unsqueeze(-1), cc, torch.zeros_like(cc))
        cl = (cc[..., 0] * nc[1] + cc[..., 1]) * nc[2] + cc[..., 2]
        k = torch.arange(mcc, device=device)
        slot = start[cl].unsqueeze(-1) + k
        valid = ((k < counts[cl].unsqueeze(-1)) & inb.unsqueeze(-1)).reshape(b - a, -1)
        cand = order[torch.where(valid, slot.reshape(b - a, -1), torch.zeros_like(valid, dtype=torch.long))]
        d = pos[ri].unsqueeze(1) - pos[cand]
        ok = valid & ((d * d).sum(-1) < r2) & (cand != ri.unsqueeze(1))
        ii, kk = ok.nonzero(as_tuple=True)
        out_i.append(ii + a)
        out_j.append(cand[ii, kk])
    pi = torch.cat(out_i)
    pj = torch.cat(out_j)
    o = torch.argsort(pi * N + pj)
    pi, pj = pi[o], pj[o]
    return pi.to(torch.int32), pj.to(torch.int32), pos[pi] - pos[pj]
