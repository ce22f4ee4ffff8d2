"""Golden vectors on the reference's own 192-atom water structure.

The reference ships one structure for this path, examples/data/water64_1x1x1_N192.data (64 H2O in a 12.4138 A cubic
box, written by ASE): the base cell its scaling runs replicate (`--base water64_1x1x1.extxyz --rep ...`,
mace_onegpu/receiver_chunk_mace.py:27).  This script reads its positions, types and box from the LAMMPS data file
and stores, for the random-init model of seed 0 (no checkpoint can be loaded here), the CPU fp64 oracle's per-atom
energies and atom forces, both with the exact radial MLP and with the 512-knot spline tables the CUDA path uses
(three-pass, chunk 64).  The reference's model code (mace-torch, e3nn, cuEquivariance) is not installed, so these
values pin the oracle against regression and give the GPU tests a fixture that needs no oracle run.

    python tests/golden/make_water64.py PATH/TO/water64_1x1x1_N192.data

writes tests/golden/water64_n192.npz next to this script.
"""
import dataclasses
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "mace-million_b200"), ROOT]

from mace_onegpu import model as M  # noqa: E402
from mace_onegpu import neighbors as NB  # noqa: E402
from mace_onegpu import structures as S  # noqa: E402
from oracle import mace_ref  # noqa: E402

TYPE_Z = {1: 8, 2: 1}     # the data file's Masses section: type 1 = O (15.999), type 2 = H (1.008)


def read_lammps_atomic(path):
    """(positions [N, 3], type ids [N], box lengths [3]) of a LAMMPS data file in `atomic` style, orthogonal box."""
    lines = open(path).read().splitlines()
    box = np.zeros(3)
    for ln in lines:
        f = ln.split()
        for d, tag in enumerate(("xlo", "ylo", "zlo")):
            if len(f) >= 4 and f[2] == tag:
                box[d] = float(f[1]) - float(f[0])
    start = next(i for i, ln in enumerate(lines) if ln.strip().startswith("Atoms"))
    rows = []
    for ln in lines[start + 1:]:
        f = ln.split()
        if not f:
            if rows:
                break
            continue
        if not f[0].lstrip("-").isdigit():
            break
        rows.append((int(f[0]), int(f[1]), float(f[2]), float(f[3]), float(f[4])))
    rows.sort()
    pos = np.array([r[2:] for r in rows])
    types = np.array([r[1] for r in rows])
    return pos, types, box


def main(path):
    pos, types, box = read_lammps_atomic(path)
    Z = np.array([TYPE_Z[t] for t in types])
    mdl = M.default_model(0)
    cols = S.species_columns(Z, mdl.arch.atomic_numbers)
    pi, pj, rij = NB.neighbor_list(pos, box, mdl.arch.r_max)
    n = len(Z)
    out = dict(pos=pos, Z=Z, box=box, n_pairs=np.int64(pi.numel()))
    for key, knots in (("exact", None), ("spline512", 512)):
        kw = {} if knots is None else dict(spline_knots=knots)
        ref = mace_ref.MaceRef(mdl.params(), dataclasses.asdict(mdl.arch), **kw)
        eat, pf = ref.three_pass(pi, pj, rij, cols, n, 64)
        out[f"eat_{key}"] = eat.numpy()
        out[f"F_{key}"] = mace_ref.atom_forces(pi, pj, pf, n).numpy()
    np.savez_compressed(os.path.join(HERE, "water64_n192.npz"), **out)
    print(f"{n} atoms, {int(pi.numel())} pairs, E = {out['eat_spline512'].sum():.6f} eV, "
          f"max|F| = {np.abs(out['F_spline512']).max():.4f} eV/A")


if __name__ == "__main__":
    main(sys.argv[1])
