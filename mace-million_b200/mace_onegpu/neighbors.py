"""Full neighbour list (both directions) of an orthorhombic periodic box or of an open point set with explicit ghost
images (input preparation for the standalone driver; the force evaluation itself takes the pair list as given, like
the ML-IAP boundary; the reference builds its standalone list in ``System.build_neighbors``,
``mace_onegpu/receiver_chunk_mace.py:114-165``).

Output convention: pairs sorted by receiver i, rij = x_i - x_j (minimum image), the edge vector of mace's
``get_edge_vectors_and_lengths`` (receiver minus sender).  On a CUDA device (and at least 3 cells per periodic
dimension) the lists come from the library's cell-list kernels (mace_b200_nbr_count / _fill, one warp per receiver,
senders of a receiver in a fixed cell-scan order).  On the host a k-d tree (scipy's cKDTree, periodic via its
``boxsize``) finds the unordered pairs, which are mirrored and sorted by (receiver, sender); it is the checker of
the CUDA lists in the tests.  ``verlet_filter`` reduces a skin list to the pairs within the cutoff at new positions
(mace_b200_verlet_filter).
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


def verlet_filter(pos, box, vrow, vj, r_cut: float, periodic: bool = True):
    """Pairs of the skin list (CSR vrow int64 [n + 1], vj int32) within r_cut at positions `pos` (CUDA; minimum
    image in `box` when periodic, plain differences for an open set with explicit ghost images): (pi int32,
    pj int32, rij fp64 [P, 3]) in the skin list's order."""
    from . import _native as N

    L = N.lib()
    st = torch.cuda.current_stream(pos.device).cuda_stream
    n = vrow.numel() - 1
    box_a = _d3(torch.as_tensor(box).tolist())
    per = 1 if periodic else 0
    counts = torch.empty(n, dtype=torch.int32, device=pos.device)
    N.check(L.mace_b200_verlet_filter(N.ptr(pos), ctypes.addressof(box_a), per, n, N.ptr(vrow), N.ptr(vj),
                                      float(r_cut), N.ptr(counts), None, None, None, None, None, st), "verlet_filter")
    rowptr = torch.zeros(n + 1, dtype=torch.int64, device=pos.device)
    rowptr[1:] = torch.cumsum(counts, 0)
    P = int(rowptr[-1].item())
    pi = torch.empty(P, dtype=torch.int32, device=pos.device)
    pj = torch.empty(P, dtype=torch.int32, device=pos.device)
    rij = torch.empty(P, 3, dtype=torch.float64, device=pos.device)
    status = torch.zeros(1, dtype=torch.int32, device=pos.device)
    N.check(L.mace_b200_verlet_filter(N.ptr(pos), ctypes.addressof(box_a), per, n, N.ptr(vrow), N.ptr(vj),
                                      float(r_cut), None, N.ptr(rowptr), N.ptr(pi), N.ptr(pj), N.ptr(rij),
                                      N.ptr(status), st), "verlet_filter")
    if int(status.item()):
        raise RuntimeError("verlet_filter: pair count changed between the count and fill passes")
    return pi, pj, rij


def _host_pairs(pos, n_recv: int, r_max: float, box=None, return_rowptr: bool = False):
    """Host pair search with a k-d tree (scipy's cKDTree; periodic when `box` is given, which needs every box
    length > 2 r_max so that each pair has exactly one image).  pos / box: fp64 CPU tensors.  Returns (pi int32,
    pj int32, rij fp64 = x_i - x_j[, rowptr int64 [n_recv + 1]]) for receivers i < n_recv and every sender j != i
    with |x_i - x_j| < r_max, sorted by (i, j)."""
    from scipy.spatial import cKDTree

    pos_np = pos.numpy()
    tree = cKDTree(pos_np, boxsize=box.numpy()) if box is not None else cKDTree(pos_np)
    ij = torch.from_numpy(tree.query_pairs(r_max, output_type="ndarray")).long()   # a < b, |d| <= r_max
    pi = torch.cat([ij[:, 0], ij[:, 1]])
    pj = torch.cat([ij[:, 1], ij[:, 0]])
    keep = pi < n_recv
    pi, pj = pi[keep], pj[keep]
    d = pos[pi] - pos[pj]
    if box is not None:
        d -= box * torch.round(d / box)
    strict = (d * d).sum(-1) < r_max * r_max                               # the kernels' strict cutoff
    pi, pj, d = pi[strict], pj[strict], d[strict]
    o = torch.argsort(pi * pos.shape[0] + pj)
    pi, pj, d = pi[o], pj[o], d[o].contiguous()
    out = (pi.to(torch.int32), pj.to(torch.int32), d)
    if return_rowptr:
        rp = torch.zeros(n_recv + 1, dtype=torch.int64)
        rp[1:] = torch.cumsum(torch.bincount(pi, minlength=n_recv), 0)
        out = out + (rp,)
    return out


def neighbor_list(pos, box, r_max: float, device="cpu", return_rowptr: bool = False):
    """Returns (pi int32 [P], pj int32 [P], rij float64 [P, 3]) for all 0 < |x_i - x_j|_mic < r_max (and the receiver
    row pointer int64 [N + 1] with return_rowptr).  CUDA device: the library's cell-list kernels; host: a periodic
    k-d tree, pairs sorted by (i, j)."""
    pos = torch.as_tensor(pos, dtype=torch.float64, device=device)
    box = torch.as_tensor(box, dtype=torch.float64, device=device)
    if not bool((box > 2.0 * r_max).all()):
        raise ValueError("minimum image needs every box length > 2 r_max")
    pos = torch.remainder(pos, box).contiguous()
    N = pos.shape[0]
    nc = torch.clamp((box / r_max).floor().long(), min=1)
    if pos.is_cuda and not bool((nc < 3).any()):
        zero = torch.zeros(3, dtype=torch.float64, device=pos.device)
        return _cuda_pairs(pos, N, zero, box / nc, nc, box, True, r_max, return_rowptr)
    pos, box = pos.cpu(), box.cpu()
    # cKDTree's periodic domain is [0, L); torch.remainder can round a tiny negative coordinate up to exactly L
    pos = torch.where(pos >= box, pos - box, pos)
    return tuple(t.to(device) for t in _host_pairs(pos, N, r_max, box, return_rowptr))


def neighbor_list_open(pos, n_recv: int, r_max: float, device="cpu", return_rowptr: bool = False):
    """Pairs of an open (non-periodic) point set with explicit ghost images: receivers are atoms [0, n_recv),
    senders any atom, 0 < |x_i - x_j| < r_max.  CUDA device: the cell-list kernels over the bounding box (cells
    >= r_max, 27 neighbours without wrap); host: a k-d tree.  Returns (pi int32, pj int32, rij fp64 = x_i - x_j)
    sorted by (pi, pj), and the receiver row pointer int64 [n_recv + 1] with return_rowptr."""
    pos = torch.as_tensor(pos, dtype=torch.float64, device=device).contiguous()
    if pos.is_cuda:
        lo = pos.min(0).values
        ext = pos.max(0).values - lo
        nc = torch.clamp((ext / r_max).floor().long(), min=1)
        width = torch.maximum(ext / nc, torch.full_like(ext, r_max))
        return _cuda_pairs(pos, n_recv, lo, width, nc, lo, False, r_max, return_rowptr)
    return _host_pairs(pos, n_recv, r_max, return_rowptr=return_rowptr)
