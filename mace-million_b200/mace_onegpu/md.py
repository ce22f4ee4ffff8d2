"""Standalone velocity-Verlet molecular dynamics on one GPU with the B200 three-pass force evaluation (the MD run of
dt = 1 fs, Verlet skin 2 A, Maxwell-Boltzmann velocities at 300 K), metal units (A, fs, eV, amu).

The pair list is a Verlet list built at r_max + skin (the library's cell-list kernels, minimum image) and filtered
to r < r_max every step by the library's Verlet-filter kernels, so the force call sees exactly the pairs LAMMPS'
ML-IAP would hand over; it is rebuilt when any atom moved more than skin / 2 since the last build.  Forces F_i = -dE/dx_i come from the pair forces dE/drij with
rij = x_i - x_j: F_i -= PF, F_j += PF.

    python -m mace_onegpu.md --config water_1m --steps 100        (prints steps/s and ns/day)
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from . import model as M
from . import neighbors as NB
from . import structures as S
from .engine import ThreePassEngine

ACC = 1.0 / 103.6427      # eV / (A amu) -> A / fs^2


class VelocityVerlet:
    def __init__(self, engine: ThreePassEngine, pos, box, elems, Z, vel, dt: float = 1.0, skin: float = 2.0):
        dev = engine.device
        self.eng = engine
        self.dt = float(dt)
        self.skin = float(skin)
        self.r_max = float(engine.model.r_max)
        self.box = torch.as_tensor(box, dtype=torch.float64, device=dev)
        self.x = torch.remainder(torch.as_tensor(pos, dtype=torch.float64, device=dev), self.box)
        self.v = torch.as_tensor(vel, dtype=torch.float64, device=dev).clone()
        m = np.array([S.MASS.get(int(z), 2.0 * int(z)) for z in Z])
        self.m = torch.as_tensor(m, dtype=torch.float64, device=dev).unsqueeze(1)
        self.elems = torch.as_tensor(elems, device=dev)
        self.n = self.x.shape[0]
        self.rebuilds = 0
        self._build()
        self.F, self.epot = self._forces()

    def _build(self):
        self.x = torch.remainder(self.x, self.box)
        pi, pj, _, vrow = NB.neighbor_list(self.x, self.box, self.r_max + self.skin, device=self.x.device,
                                           return_rowptr=True)
        self.vpi, self.vpj, self.vrow = pi, pj, vrow
        self.x_ref = self.x.clone()
        self.rebuilds += 1

    def _pairs(self):
        """Pairs within r_max at the current positions, from the Verlet list."""
        if self.x.is_cuda:
            return NB.verlet_filter(self.x, self.box, self.vrow, self.vpj, self.r_max)
        vpi, vpj = self.vpi.long(), self.vpj.long()
        d = self.x[vpi] - self.x[vpj]
        d = d - self.box * torch.round(d / self.box)
        keep = (d * d).sum(1) < self.r_max * self.r_max
        return self.vpi[keep], self.vpj[keep], d[keep]

    def _forces(self):
        pi, pj, rij = self._pairs()
        plan = self.eng.plan(pi, pj, rij, self.elems, self.n, self.n)
        pi, pj = pi.long(), pj.long()
        eat, pf = self.eng.evaluate(plan)
        F = torch.zeros_like(self.x)
        F.index_add_(0, pi, -pf)
        F.index_add_(0, pj, pf)
        return F, float(eat.sum())

    def kinetic(self) -> float:
        return float(0.5 * (self.m * self.v * self.v).sum() / ACC)

    def step(self):
        self.v += 0.5 * self.dt * ACC * self.F / self.m
        self.x += self.dt * self.v
        disp = self.x - self.x_ref
        disp = disp - self.box * torch.round(disp / self.box)
        if float((disp * disp).sum(1).max()) > (0.5 * self.skin) ** 2:
            self._build()
        self.F, self.epot = self._forces()
        self.v += 0.5 * self.dt * ACC * self.F / self.m


class DomainVelocityVerlet(VelocityVerlet):
    """Velocity Verlet on N GPUs over spatial domains (one process per GPU, torch.distributed).

    Every rank keeps all positions, velocities and forces of the system: they are replicated and stay bitwise
    identical on all ranks. Each rank evaluates only the forces of its own domain's atoms: local receivers, local
    or ghost senders, with the H1 / G1 halo exchanges of domain.HaloExchange. One all-reduce of the [N, 3] force
    array (and of the energy) per step then gives every rank every force, and each rank integrates all atoms.

    The decomposition (owners, ghost images within r_max + skin, exchange maps) and the Verlet lists (r_max + skin)
    are rebuilt together, on the device (domain.DeviceDecomposition), when any atom has moved more than skin / 2
    since the last build. Between rebuilds ownership and the ghost sets stay fixed, as between LAMMPS
    reneighborings: a pair within r_max now was within r_max + skin of a receiver inside its domain at the build.
    The rebuild decision needs no communication, because all ranks see the same positions.

    engine: anything with the ThreePassEngine calls used here (device, model.r_max, plan, evaluate).
    overlap: run the exchanges overlapped with interior chunks (evaluate(plan, halo=...)), else between the passes.
    """

    def __init__(self, engine, pos, box, elems, Z, vel, grid, rank: int, dt: float = 1.0, skin: float = 2.0,
                 overlap: bool = True, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.grid, self.rank, self.overlap = tuple(int(g) for g in grid), int(rank), bool(overlap)
        super().__init__(engine, pos, box, elems, Z, vel, dt=dt, skin=skin)

    def _build(self):
        from . import domain as DM

        self.x = torch.remainder(self.x, self.box)
        dec = DM.DeviceDecomposition(self.x, self.box, self.grid, self.r_max + self.skin)
        p, gid, nl = dec.rank_atoms(self.rank)
        self.dec, self.gid, self.nl = dec, gid, nl
        self.cols = self.elems[gid]
        self.hx = DM.HaloExchange(dec, self.rank, self.x.device, group=self.group)
        _, self.vpj, _, self.vrow = NB.neighbor_list_open(p, nl, self.r_max + self.skin, device=self.x.device,
                                                          return_rowptr=True)
        self.x_ref = self.x.clone()
        self.rebuilds += 1

    def _pairs(self):
        """Pairs within r_max at the current positions: local atoms and the fixed ghost images, no wrap."""
        p, _, _ = self.dec.rank_atoms(self.rank, pos=self.x)
        if p.is_cuda:
            return NB.verlet_filter(p, self.box, self.vrow, self.vpj, self.r_max, periodic=False)
        rows = torch.repeat_interleave(torch.arange(self.nl, device=p.device), self.vrow[1:] - self.vrow[:-1])
        vpj = self.vpj.long()
        d = p[rows] - p[vpj]
        keep = (d * d).sum(1) < self.r_max * self.r_max
        return rows[keep].to(torch.int32), self.vpj[keep], d[keep]

    def _forces(self):
        pi, pj, rij = self._pairs()
        nt = int(self.gid.numel())
        plan = self.eng.plan(pi, pj, rij, self.cols, self.nl, nt)
        if self.overlap:
            eat, pf = self.eng.evaluate(plan, halo=self.hx)
        else:
            eat, pf = self.eng.evaluate(plan, self.hx.forward, self.hx.reverse)
        Fl = torch.zeros(nt, 3, dtype=torch.float64, device=self.x.device)
        Fl.index_add_(0, pi.long(), -pf)
        Fl.index_add_(0, pj.long(), pf)
        F = torch.zeros_like(self.x)
        F.index_add_(0, self.gid, Fl)                   # ghost images add onto the atoms they copy
        e = eat.double().sum().reshape(1)
        self.dist.all_reduce(F, group=self.group)
        self.dist.all_reduce(e, group=self.group)
        return F, float(e.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="water_1m", choices=["water_1m", "water_24k", "water_192"])
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--dt", type=float, default=1.0)
    ap.add_argument("--skin", type=float, default=2.0)
    ap.add_argument("--temperature", type=float, default=300.0)
    ap.add_argument("--chunk", type=int, default=16384)
    a = ap.parse_args()
    n = {"water_1m": 70, "water_24k": 20, "water_192": 4}[a.config]
    dev = torch.device("cuda")
    mdl = M.default_model(0)
    pos, Z, box = S.water_box(n, seed=0)
    cols = S.species_columns(Z, mdl.arch.atomic_numbers)
    vel = S.maxwell_boltzmann(Z, a.temperature, seed=0)
    eng = ThreePassEngine(mdl, sorted(set(cols.tolist())), chunk=a.chunk, device=dev)
    md = VelocityVerlet(eng, pos, box, cols, Z, vel, dt=a.dt, skin=a.skin)
    e0 = md.epot + md.kinetic()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        md.step()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    e1 = md.epot + md.kinetic()
    sps = a.steps / dt
    print(json.dumps({"config": a.config, "atoms": len(Z), "steps": a.steps, "dt_fs": a.dt, "seconds": dt,
                      "steps_per_s": sps, "ns_per_day": sps * a.dt * 86400 / 1e6, "atom_steps_per_s": sps * len(Z),
                      "neighbour_rebuilds": md.rebuilds, "energy_drift_eV_per_atom": (e1 - e0) / len(Z)}))


if __name__ == "__main__":
    main()
