"""Full neighbour list (both directions) of an orthorhombic periodic box: cell list + minimum image, in torch so that
it runs on the host or on the GPU (input preparation for the standalone driver; the force evaluation itself takes the
pair list as given, like the ML-IAP boundary).  The algorithm is the one of the reference's
``System.build_neighbors`` (``mace_onegpu/receiver_chunk_mace.py:114-165``): 27-cell candidates per atom, a count
pass then a fill pass, brute force when a box dimension holds fewer than 3 cells.

Output convention: pairs sorted by receiver i (then by sender j), rij = x_i - x_j (minimum image), the edge vector of
mace's ``get_edge_vectors_and_lengths`` (receiver minus sender).
"""
from __future__ import annotations

import torch


def neighbor_list(pos, box, r_max: float, device="cpu", block: int = 16384):
    """Returns (pi int32 [P], pj int32 [P], rij float64 [P, 3]) for all 0 < |x_i - x_j|_mic < r_max."""
    pos = torch.as_tensor(pos, dtype=torch.float64, device=device)
    box = torch.as_tensor(box, dtype=torch.float64, device=device)
    if not bool((box > 2.0 * r_max).all()):
        raise ValueError("minimum image needs every box length > 2 r_max")
    pos = torch.remainder(pos, box)
    N = pos.shape[0]
    r2 = r_max * r_max
    nc = torch.clamp((box / r_max).floor().long(), min=1)
    brute = bool((nc < 3).any())
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
    return pi.to(torch.int32), pj.to(torch.int32), rij


def neighbor_list_open(pos, n_recv: int, r_max: float, device="cpu", block: int = 16384):
    """Pairs of an open (non-periodic) point set with explicit ghost images: receivers are atoms [0, n_recv),
    senders any atom, 0 < |x_i - x_j| < r_max.  Cell list over the bounding box (cells >= r_max, 27 neighbours
    without wrap).  Returns (pi int32, pj int32, rij fp64 = x_i - x_j) sorted by (pi, pj)."""
    pos = torch.as_tensor(pos, dtype=torch.float64, device=device)
    N = pos.shape[0]
    lo = pos.min(0).values
    ext = pos.max(0).values - lo
    nc = torch.clamp((ext / r_max).floor().long(), min=1)
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
