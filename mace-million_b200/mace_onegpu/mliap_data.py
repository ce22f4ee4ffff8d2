"""A standalone ML-IAP data object: the driver side of the ``pair_style mliap unified`` boundary for runs without
LAMMPS (tests, the standalone driver and the end-to-end benchmark).

It carries what LAMMPS' MLIAPDataKokkosDevice hands to ``compute_forces`` (nlocal, ntotal, npairs, elems, pair_i,
pair_j, rij, eatoms, energy) and implements the three callbacks with LAMMPS' semantics:
* forward_exchange(src, dst, D): dst = src with every ghost row replaced by its owner's row;
* reverse_exchange(src, dst, D): dst = src with every ghost row added onto its owner's row (ghost rows of dst = 0);
* update_pair_forces_gpu(PF): keeps the pair forces dE/drij (optionally copied to host memory, as LAMMPS reads them
  into its force array) and, when positions are known, accumulates atom forces.
Ghost atoms are described by an owner map (owner[j] = local atom of which ghost j is a periodic image).
"""
from __future__ import annotations

import torch


class MLIAPData:
    def __init__(self, pair_i, pair_j, rij, elems, nlocal: int, owner=None, host_outputs: bool = False,
                 exchange=None):
        self.pair_i = pair_i
        self.pair_j = pair_j
        self.rij = rij
        self.elems = elems
        self.nlocal = int(nlocal)
        self.ntotal = int(elems.shape[0])
        self.npairs = int(pair_i.shape[0])
        dev = rij.device
        pin = host_outputs and not rij.is_cuda and torch.cuda.is_available()
        self.eatoms = torch.zeros(self.nlocal, dtype=torch.float64, device=dev, pin_memory=pin)
        self.energy = 0.0
        self.host_outputs = host_outputs
        self.pair_forces = None
        self._pf_host = torch.empty((self.npairs, 3), dtype=torch.float64, pin_memory=pin) if host_outputs else None
        # pinned host destination a force evaluation may fill directly, chunk by chunk (overlapped D2H)
        self.pair_forces_host = self._pf_host if pin else None
        self.owner = None if owner is None else torch.as_tensor(owner).long()
        self._owner_dev = {}
        self.exchange = exchange          # distributed halo exchange (forward(H) / reverse(G) in place), e.g. domain.py

    def _own(self, device):
        o = self._owner_dev.get(device)
        if o is None:
            o = self.owner.to(device)
            self._owner_dev[device] = o
        return o

    def forward_exchange(self, src, dst, D):
        dst.copy_(src)
        if self.exchange is not None:
            self.exchange.forward(dst)
        elif self.owner is not None and self.ntotal > self.nlocal:
            own = self._own(src.device)
            dst[self.nlocal:] = src[own[self.nlocal:]]

    def reverse_exchange(self, src, dst, D):
        dst.copy_(src)
        if self.exchange is not None:
            self.exchange.reverse(dst)
        elif self.owner is not None and self.ntotal > self.nlocal:
            own = self._own(src.device)
            dst.index_add_(0, own[self.nlocal:], src[self.nlocal:])
            dst[self.nlocal:] = 0

    def update_pair_forces_gpu(self, PF):
        if self.host_outputs:
            if PF is not self._pf_host:             # else already written there by the evaluation
                self._pf_host.copy_(PF, non_blocking=True)
            self.pair_forces = self._pf_host
        else:
            self.pair_forces = PF

    def atom_forces(self):
        """F = -dE/dx with rij = x_i - x_j (the model's edge vector): F_i -= PF, F_j += PF; ghosts folded onto owners."""
        PF = torch.as_tensor(self.pair_forces).double().cpu()
        pi = torch.as_tensor(self.pair_i).long().cpu()
        pj = torch.as_tensor(self.pair_j).long().cpu()
        F = torch.zeros(self.ntotal, 3, dtype=torch.float64)
        F.index_add_(0, pi, -PF)
        F.index_add_(0, pj, PF)
        if self.owner is not None and self.ntotal > self.nlocal:
            F[: self.nlocal].index_add_(0, self.owner[self.nlocal:], F[self.nlocal:])
        return F[: self.nlocal]


def from_structure(pos, Z, box, model, r_max=None, device="cpu", host_outputs=False):
    """ML-IAP data of a periodic box with the minimum-image pair list (no ghosts)."""
    from . import neighbors, structures

    r_max = float(model.r_max if r_max is None else r_max)
    pi, pj, rij = neighbors.neighbor_list(pos, box, r_max, device=device)
    cols = torch.as_tensor(structures.species_columns(Z, model.atomic_numbers.tolist()), device=device)
    return MLIAPData(pi, pj, rij, cols, len(Z), host_outputs=host_outputs)
