"""Seeded synthetic structures of the benchmark configurations (no public dataset is used; the structures are
procedural).  Water: H2O molecules (O-H 0.9572 A, H-O-H 104.52 deg) with uniformly random orientations, the O atom of
each molecule on a cubic grid (spacing 3.104 A) jittered by N(0, 0.05 A), periodic cubic box.  Alloy: bcc lattice
(a = 3.0 A) with N(0, 0.1 A) displacements and a uniformly drawn element per site.

Species are returned as atomic numbers; ``species_columns`` maps them to the model's one-hot columns.
"""
from __future__ import annotations

import math

import numpy as np

WATER_SPACING = 3.104
ALLOY_Z = (3, 8, 11, 12, 13, 14, 16, 20, 22, 26, 27, 28, 29, 30, 40, 42)
MASS = {1: 1.008, 3: 6.94, 8: 15.999, 11: 22.990, 12: 24.305, 13: 26.982, 14: 28.085, 16: 32.06, 20: 40.078,
        22: 47.867, 26: 55.845, 27: 58.933, 28: 58.693, 29: 63.546, 30: 65.38, 40: 91.224, 42: 95.95}   # amu


def _random_rotations(rng: np.random.Generator, n: int) -> np.ndarray:
    q = rng.normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    return np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], -1),
        np.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], -1),
        np.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], -1)], 1)


def water_box(nx: int, ny: int | None = None, nz: int | None = None, seed: int = 0,
              spacing: float = WATER_SPACING, jitter: float = 0.05):
    """(positions fp64 [3 n_mol, 3], atomic numbers int [3 n_mol] (O, H, H per molecule), box fp64 [3])."""
    ny = nx if ny is None else ny
    nz = nx if nz is None else nz
    rng = np.random.default_rng(seed)
    g = np.stack(np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij"), -1).reshape(-1, 3)
    n = g.shape[0]
    centre = g * spacing + rng.normal(scale=jitter, size=(n, 3))
    half = math.radians(104.52) / 2.0
    d = 0.9572
    body = np.array([[0.0, 0.0, 0.0], [d * math.sin(half), d * math.cos(half), 0.0],
                     [-d * math.sin(half), d * math.cos(half), 0.0]])
    R = _random_rotations(rng, n)
    pos = centre[:, None, :] + np.einsum("nij,aj->nai", R, body)
    box = np.array([nx, ny, nz], dtype=np.float64) * spacing
    Z = np.tile(np.array([8, 1, 1], dtype=np.int64), n)
    return np.remainder(pos.reshape(-1, 3), box), Z, box


def alloy_bcc(n: int = 60, a: float = 3.0, seed: int = 0, disp: float = 0.1, zs=ALLOY_Z):
    rng = np.random.default_rng(seed)
    g = np.stack(np.meshgrid(np.arange(n), np.arange(n), np.arange(n), indexing="ij"), -1).reshape(-1, 3)
    base = np.concatenate([g, g + 0.5], 0) * a
    pos = base + rng.normal(scale=disp, size=base.shape)
    box = np.full(3, n * a)
    Z = np.asarray(zs, dtype=np.int64)[rng.integers(0, len(zs), size=pos.shape[0])]
    return np.remainder(pos, box), Z, box


def tile(pos, Z, box, reps):
    """Periodic replica of a box: reps = (rx, ry, rz) copies along each axis.  Atom k of copy c = (cx, cy, cz) (copies
    in C order, z fastest) gets index c * n + k and position pos[k] + c * box, so every replica atom's environment is
    its image's environment in the original periodic box."""
    pos = np.asarray(pos, dtype=np.float64)
    box = np.asarray(box, dtype=np.float64)
    shifts = np.stack(np.meshgrid(*[np.arange(r) for r in reps], indexing="ij"), -1).reshape(-1, 3) * box
    P = (shifts[:, None, :] + pos[None, :, :]).reshape(-1, 3)
    return P, np.tile(np.asarray(Z), len(shifts)), box * np.asarray(reps, dtype=np.float64)


def _spread3(v: np.ndarray) -> np.ndarray:
    """Bits of v (< 2^21) moved to every third position (bit b -> bit 3 b)."""
    v = v.astype(np.uint64) & np.uint64(0x1FFFFF)
    for shift, mask in ((32, 0x1F00000000FFFF), (16, 0x1F0000FF0000FF), (8, 0x100F00F00F00F00F),
                        (4, 0x10C30C30C30C30C3), (2, 0x1249249249249249)):
        v = (v | (v << np.uint64(shift))) & np.uint64(mask)
    return v


def morton_order(pos, box, cell: float = 3.0) -> np.ndarray:
    """Permutation that sorts atoms along a Z-order (Morton) curve of cubic cells of about `cell` A, atoms of one cell
    keeping their relative order.  Spatially sorted atoms are what a production MD engine passes (LAMMPS re-sorts
    atoms spatially every 1000 steps by default; the reference's standalone driver orders them on a Morton curve
    too, mace_onegpu/receiver_chunk_mace.py:100-104): receivers that are close in index then share senders, so
    the senders' feature rows are reused from L2."""
    pos = np.remainder(np.asarray(pos, dtype=np.float64), box)
    nc = np.maximum(np.floor(np.asarray(box) / cell).astype(np.int64), 1)
    c = np.minimum((pos / (np.asarray(box) / nc)).astype(np.int64), nc - 1)
    code = (_spread3(c[:, 0]) << np.uint64(2)) | (_spread3(c[:, 1]) << np.uint64(1)) | _spread3(c[:, 2])
    return np.argsort(code, kind="stable")


def lammps_bin_order(pos, box, binsize: float = 3.5) -> np.ndarray:
    """Permutation into the order of LAMMPS's spatial atom sort (atom_modify sort, on by default every 1000 steps):
    cubic-ish bins of about `binsize` A (LAMMPS's default is half the neighbour cutoff, (5 + 2) / 2 A for a 5 A
    model with a 2 A skin), numbered x fastest, then y, then z; atoms of one bin keep their relative order.  A
    chunk of consecutive receivers is then a slab a few bins thick, whose senders lie in the neighbouring slabs."""
    pos = np.remainder(np.asarray(pos, dtype=np.float64), box)
    nb = np.maximum(np.floor(np.asarray(box) / binsize).astype(np.int64), 1)
    c = np.minimum((pos / (np.asarray(box) / nb)).astype(np.int64), nb - 1)
    return np.argsort((c[:, 2] * nb[1] + c[:, 1]) * nb[0] + c[:, 0], kind="stable")


def species_columns(Z, atomic_numbers) -> np.ndarray:
    """Model one-hot column of every atom (index into atomic_numbers)."""
    lut = {int(z): i for i, z in enumerate(atomic_numbers)}
    return np.array([lut[int(z)] for z in np.asarray(Z)], dtype=np.int64)


def maxwell_boltzmann(Z, temperature: float, seed: int = 0) -> np.ndarray:
    """Velocities (A/fs) at the given temperature with zero total momentum."""
    kB = 8.617333262e-5                                    # eV / K
    amu = 103.6427                                         # 1 amu A^2 / fs^2 = 103.6427 eV
    m = np.array([MASS.get(int(z), 2.0 * int(z)) for z in Z]) * amu
    rng = np.random.default_rng(seed)
    v = rng.normal(size=(len(Z), 3)) * np.sqrt(kB * temperature / m)[:, None]
    v -= (m[:, None] * v).sum(0) / m.sum()
    return v
