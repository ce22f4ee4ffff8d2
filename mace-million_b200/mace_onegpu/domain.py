"""Spatial domain decomposition of a periodic orthorhombic box over ranks, with explicit ghost atoms and the two halo
exchanges of the three-pass evaluation (H1 forward: owner rows -> ghost rows; G1 reverse: ghost rows summed onto
owners) over torch.distributed point-to-point (NCCL on GPUs, gloo on CPU).

The reference delegates this to LAMMPS (MPI ranks, ghost comm through data.forward_exchange / reverse_exchange,
``mace_onegpu/mliap_threepass.py:40-55, 522, 556``).  Standalone, every rank generates the same global structure and
computes the same decomposition, so the send / receive maps need no communication:
* rank r of a grid (px, py, pz) owns the atoms whose wrapped position falls in its block;
* its ghosts are the periodic images of atoms (its own included) that fall within `r_ghost` outside its block;
* ghost rows are ordered by (owner rank, owner's local index, image), i.e. one contiguous block per owner rank, and
  the owner's send list to r is the owner-local indices of that block in the same order.
Forward exchange: pack owner rows -> send; receive straight into the contiguous ghost block.  Reverse exchange: send
the contiguous ghost block; receive into a buffer and scatter-add onto the owner rows (a CUDA kernel on GPUs).
"""
from __future__ import annotations

import itertools

import numpy as np
import torch


def grid_for(world: int):
    return {1: (1, 1, 1), 2: (2, 1, 1), 4: (2, 2, 1), 8: (2, 2, 2)}.get(world) or _factor3(world)


def _factor3(n):
    best = None
    for a in range(1, n + 1):
        if n % a:
            continue
        for b in range(1, n // a + 1):
            if (n // a) % b:
                continue
            c = n // a // b
            key = max(a, b, c)
            if best is None or key < best[0]:
                best = (key, (a, b, c))
    return best[1]


class Decomposition:
    """All ranks' local / ghost sets of a periodic box (numpy, computed identically on every rank)."""

    def __init__(self, pos, box, grid, r_ghost: float):
        pos = np.remainder(np.asarray(pos, dtype=np.float64), box)
        box = np.asarray(box, dtype=np.float64)
        grid = np.asarray(grid, dtype=np.int64)
        self.box, self.grid, self.r_ghost = box, grid, float(r_ghost)
        self.nranks = int(grid.prod())
        w = box / grid
        if np.any(w < 1e-9):
            raise ValueError("empty domain")
        cell = np.minimum((pos / w).astype(np.int64), grid - 1)
        owner = (cell[:, 0] * grid[1] + cell[:, 1]) * grid[2] + cell[:, 2]
        self.owner = owner
        # ghost entries (rank, global atom, image shift) over all ranks
        entries = []
        for s in itertools.product((-1, 0, 1), repeat=3):
            s = np.asarray(s)
            q = pos + s * box
            near = np.all((q > -r_ghost) & (q < box + r_ghost), axis=1)
            if not near.any():
                continue
            ids = np.nonzero(near)[0]
            qq = q[ids]
            dlo = np.clip(np.floor((qq - r_ghost) / w).astype(np.int64), 0, grid - 1)
            dhi = np.clip(np.floor((qq + r_ghost) / w).astype(np.int64), 0, grid - 1)
            span = int(np.max(dhi - dlo)) + 1
            for off in itertools.product(range(span), repeat=3):
                d = dlo + np.asarray(off)
                okd = np.all(d <= dhi, axis=1)
                if not okd.any():
                    continue
                dd = d[okd]
                ii = ids[okd]
                qd = qq[okd]
                lo = dd * w
                hi = lo + w
                inside_ext = np.all((qd >= lo - r_ghost) & (qd < hi + r_ghost), axis=1)
                inside = np.all((qd >= lo) & (qd < hi), axis=1)
                rank = (dd[:, 0] * grid[1] + dd[:, 1]) * grid[2] + dd[:, 2]
                keep = inside_ext & ~(inside & (not s.any()))
                if keep.any():
                    code = (s[0] + 1) * 9 + (s[1] + 1) * 3 + s[2] + 1
                    entries.append(np.stack([rank[keep], ii[keep], np.full(int(keep.sum()), code)], 1))
        E = np.concatenate(entries, 0) if entries else np.zeros((0, 3), dtype=np.int64)
        E = np.unique(E, axis=0)                                   # (rank, atom, image) unique
        # each rank's atoms: interior atoms (a ghost on no rank, so no ghost lies within r_ghost > r_max of them)
        # first, boundary atoms (sent to some rank) last, each group in global order.  Interior receivers have no
        # ghost senders, so their chunks can run while a halo exchange is in flight.
        boundary = np.zeros(len(pos), dtype=bool)
        boundary[E[:, 1]] = True
        key = owner * 2 + boundary
        order = np.argsort(key, kind="stable")
        counts = np.bincount(owner, minlength=self.nranks)
        self.local = np.split(order, np.cumsum(counts)[:-1])          # global indices of each rank's atoms
        self.n_interior = [int((~boundary[idx]).sum()) for idx in self.local]
        local_index = np.empty(len(pos), dtype=np.int64)
        for r, idx in enumerate(self.local):
            local_index[idx] = np.arange(len(idx))
        self.local_index = local_index
        self.ghost = []
        for r in range(self.nranks):
            er = E[E[:, 0] == r]
            own = self.owner[er[:, 1]]
            key = np.lexsort((er[:, 2], self.local_index[er[:, 1]], own))
            self.ghost.append(er[key, 1:])                         # [n_ghost, (global atom, image code)]
        self.pos = pos

    def image_shift(self, code):
        code = np.asarray(code)
        s = np.stack([code // 9 - 1, (code // 3) % 3 - 1, code % 3 - 1], -1)
        return s * self.box

    def rank_atoms(self, r):
        """(positions [nl + ng, 3] with ghosts at their image positions, global atom ids, nl)."""
        loc = self.local[r]
        gh = self.ghost[r]
        p = np.concatenate([self.pos[loc], self.pos[gh[:, 0]] + self.image_shift(gh[:, 1])], 0)
        return p, np.concatenate([loc, gh[:, 0]]), len(loc)

    def recv_blocks(self, r):
        """{owner rank: (start, stop)} ghost-row ranges of rank r (row index counted from nl)."""
        gh = self.ghost[r]
        own = self.owner[gh[:, 0]]
        out = {}
        for o in np.unique(own):
            ids = np.nonzero(own == o)[0]
            out[int(o)] = (int(ids[0]), int(ids[-1]) + 1)
        return out

    def send_list(self, r, p):
        """Owner-local indices (on rank r) of the ghost block rank p receives from r, in p's ghost order."""
        gh = self.ghost[p]
        sel = self.owner[gh[:, 0]] == r
        return self.local_index[gh[sel, 0]]


class DeviceDecomposition:
    """The same decomposition as ``Decomposition`` (same owners, local order, ghost sets and ghost order), computed
    with torch on the positions' device, so that a GPU builds it for millions of atoms in well under a second (the
    numpy construction takes about a minute per 2M atoms): the multi-GPU bench and the MD driver, which rebuilds it
    whenever the Verlet lists are rebuilt.  Index arrays are int64 tensors on that device; ``local`` and ``ghost`` are
    per-rank lists of them.

    Every (rank, atom, image) ghost entry is packed into one int64 key, (rank * N + atom) * 27 + image code, so the
    deduplication and the (owner rank, owner-local index, image) ghost order are single sorts."""

    def __init__(self, pos, box, grid, r_ghost: float):
        pos = torch.as_tensor(pos, dtype=torch.float64)
        dev = pos.device
        box = torch.as_tensor(box, dtype=torch.float64).to(dev)      # numpy, list or tensor on any device
        pos = torch.remainder(pos, box)
        g = torch.as_tensor(np.asarray(grid, dtype=np.int64), device=dev)
        self.box, self.r_ghost, self.device = box, float(r_ghost), dev
        self.grid = np.asarray(grid, dtype=np.int64)
        self.nranks = int(self.grid.prod())
        n = pos.shape[0]
        w = box / g
        if bool((w < 1e-9).any()):
            raise ValueError("empty domain")
        gm1 = g - 1
        rg = self.r_ghost

        def linear(c):
            return (c[:, 0] * g[1] + c[:, 1]) * g[2] + c[:, 2]

        cell = torch.minimum(torch.floor(pos / w).long(), gm1)
        self.owner = linear(cell)
        keys = []
        for s in itertools.product((-1, 0, 1), repeat=3):
            st = torch.tensor(s, dtype=torch.float64, device=dev)
            q = pos + st * box
            near = ((q > -rg) & (q < box + rg)).all(1)
            ids = torch.nonzero(near).squeeze(1)
            if ids.numel() == 0:
                continue
            qq = q[ids]
            dlo = torch.clamp(torch.floor((qq - rg) / w).long(), min=0).minimum(gm1)
            dhi = torch.clamp(torch.floor((qq + rg) / w).long(), min=0).minimum(gm1)
            span = int((dhi - dlo).max()) + 1
            code = (s[0] + 1) * 9 + (s[1] + 1) * 3 + s[2] + 1
            for off in itertools.product(range(span), repeat=3):
                d = dlo + torch.tensor(off, dtype=torch.int64, device=dev)
                okd = (d <= dhi).all(1)
                dd, ii, qd = d[okd], ids[okd], qq[okd]
                lo = dd.double() * w
                hi = lo + w
                keep = ((qd >= lo - rg) & (qd < hi + rg)).all(1)
                if not any(s):
                    keep &= ~((qd >= lo) & (qd < hi)).all(1)
                if bool(keep.any()):
                    keys.append((linear(dd[keep]) * n + ii[keep]) * 27 + code)
        E = torch.unique(torch.cat(keys)) if keys else torch.zeros(0, dtype=torch.int64, device=dev)
        e_rank, e_atom, e_code = E // (27 * n), (E // 27) % n, E % 27
        boundary = torch.zeros(n, dtype=torch.bool, device=dev)
        boundary[e_atom] = True
        # local atoms: interior first, then boundary atoms, each group in global order (as Decomposition)
        order = torch.sort(self.owner * 2 + boundary.long(), stable=True).indices
        counts = torch.bincount(self.owner, minlength=self.nranks).tolist()
        self.local = list(torch.split(order, counts))
        self.n_interior = [int((~boundary[idx]).sum()) for idx in self.local]
        local_index = torch.empty(n, dtype=torch.int64, device=dev)
        for idx in self.local:
            local_index[idx] = torch.arange(idx.numel(), device=dev)
        self.local_index = local_index
        self.ghost = []
        for r in range(self.nranks):
            sel = e_rank == r
            a, c = e_atom[sel], e_code[sel]
            k = torch.sort((self.owner[a] * n + local_index[a]) * 27 + c).indices
            self.ghost.append(torch.stack([a[k], c[k]], 1))          # [n_ghost, (global atom, image code)]
        self.pos = pos

    def image_shift(self, code):
        code = torch.as_tensor(code, device=self.device)
        s = torch.stack([code // 9 - 1, (code // 3) % 3 - 1, code % 3 - 1], -1)
        return s.double() * self.box

    def rank_atoms(self, r, pos=None):
        """(positions [nl + ng, 3] with ghosts at their image positions, global atom ids, nl); `pos` replaces the
        positions the decomposition was built from (same atoms, e.g. later MD positions)."""
        pos = self.pos if pos is None else pos
        loc, gh = self.local[r], self.ghost[r]
        p = torch.cat([pos[loc], pos[gh[:, 0]] + self.image_shift(gh[:, 1])], 0)
        return p, torch.cat([loc, gh[:, 0]]), int(loc.numel())

    def recv_blocks(self, r):
        """{owner rank: (start, stop)} ghost-row ranges of rank r (row index counted from nl)."""
        own = self.owner[self.ghost[r][:, 0]]
        uniq, cnt = torch.unique_consecutive(own, return_counts=True)
        out, start = {}, 0
        for o, c in zip(uniq.tolist(), cnt.tolist()):
            out[int(o)] = (start, start + int(c))
            start += int(c)
        return out

    def send_list(self, r, p):
        """Owner-local indices (on rank r) of the ghost block rank p receives from r, in p's ghost order."""
        gh = self.ghost[p]
        return self.local_index[gh[self.owner[gh[:, 0]] == r, 0]]


class HaloExchange:
    """The H1 forward / G1 reverse exchanges of one rank for feature rows [nt, D] (torch.distributed P2P)."""

    def __init__(self, dec: Decomposition, rank: int, device, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = rank
        self.device = torch.device(device)
        self.nl = len(dec.local[rank])
        self.recv = dec.recv_blocks(rank)                                       # owner -> (g0, g1)
        self.send = {}
        for p in range(dec.nranks):
            idx = dec.send_list(rank, p)
            if len(idx):
                self.send[p] = torch.as_tensor(idx, dtype=torch.int32, device=self.device)
        self.bytes_fwd = 0
        self._bufs = {}
        self._pending = []
        self.n_interior = dec.n_interior[rank]      # local atoms [0, n_interior) have no ghost neighbours

    def _buf(self, key, n, D, dtype):
        b = self._bufs.get(key)
        if b is None or b.shape[0] < n or b.shape[1] != D or b.dtype != dtype:
            b = torch.empty(max(n, 1), D, dtype=dtype, device=self.device)
            self._bufs[key] = b
        return b[:n]

    def _pack(self, src, idx, out=None):
        """Rows src[idx] (into `out` when given, else a new buffer)."""
        if src.is_cuda:
            from . import _native as N

            if out is None:
                return N.ops().pack_halo(src, idx)
            st = torch.cuda.current_stream(src.device).cuda_stream
            N.check(N.lib().mace_b200_pack_rows(N.ptr(src), N.ptr(idx), idx.numel(), src.shape[1], N.ptr(out), st),
                    "pack_rows")
            return out
        if out is None:
            return src[idx.long()]
        out.copy_(src[idx.long()])
        return out

    def _unpack_add(self, buf, idx, dst):
        if dst.is_cuda:
            from . import _native as N

            N.ops().unpack_halo_add(dst, buf, idx)
        else:
            dst.index_add_(0, idx.long(), buf)

    def forward(self, H):
        """H [nt, D]: ghost rows <- owner rows (in place)."""
        dist = self.dist
        ops = []
        self._sent = []
        for p, idx in self.send.items():
            if p == self.rank:
                g0, g1 = self.recv[p]
                self._pack(H, idx, H[self.nl + g0:self.nl + g1])
                continue
            buf = self._pack(H, idx)
            self._sent.append(buf)                      # alive until the grouped send completes
            ops.append(dist.P2POp(dist.isend, buf, p, group=self.group))
        for o, (g0, g1) in self.recv.items():
            if o != self.rank:
                ops.append(dist.P2POp(dist.irecv, H[self.nl + g0:self.nl + g1], o, group=self.group))
        self._run(ops)
        self._sent = []

    def reverse(self, G):
        """G [nt, D]: owner rows += ghost rows (ghost rows left as they are)."""
        self.reverse_comm(G)
        self.reverse_unpack(G)

    def reverse_comm(self, G):
        """The communication half of reverse(): ghost rows go to their owners, the owners' received blocks wait in
        buffers (and the rank's own periodic images in a copy) until reverse_unpack(G) adds them."""
        dist = self.dist
        D = G.shape[1]
        ops, pending = [], []
        for o, (g0, g1) in self.recv.items():
            if o == self.rank:
                continue
            ops.append(dist.P2POp(dist.isend, G[self.nl + g0:self.nl + g1].contiguous(), o, group=self.group))
        for p, idx in self.send.items():
            if p == self.rank:
                continue
            buf = self._buf(("r", p), idx.numel(), D, G.dtype)
            ops.append(dist.P2POp(dist.irecv, buf, p, group=self.group))
            pending.append((buf, idx))
        self._run(ops)
        if self.rank in self.send:
            g0, g1 = self.recv[self.rank]
            pending.append((G[self.nl + g0:self.nl + g1].clone(), self.send[self.rank]))
        self._pending = pending

    def reverse_unpack(self, G):
        """Adds the blocks reverse_comm(G) received onto their owner rows (on the current stream, which may differ
        from the one reverse_comm ran on: the buffers are recorded on it before they are released)."""
        for buf, idx in self._pending:
            self._unpack_add(buf, idx, G)
            if buf.is_cuda:
                buf.record_stream(torch.cuda.current_stream(buf.device))
        self._pending = []

    def _run(self, ops):
        if not ops:
            return
        for w in self.dist.batch_isend_irecv(ops):
            w.wait()
