"""TEST INFRASTRUCTURE (oracle): O(3) constants computed by an independent route.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may import this package; it is the checker of
the CUDA path, never part of it.

Conventions (shared with the product, computed differently here):
* real SH, l <= 3, e3nn 0.4 polynomial forms, component normalisation (sum_m Y_lm^2 = 2l+1);
* Wigner-3j in that basis, unit Frobenius norm, first non-zero entry (C order) positive.
Route: exact complex 3j symbols (sympy.physics.wigner.wigner_3j) mapped to the real basis with the matrix Q_l fitted
between our real SH and scipy's complex SH (Y_real = Q_l Y_complex); for l > 3 (intermediate couplings only) the real
basis is the standard real combination of complex SH, whose convention cancels in every contracted coupling.
"""
from __future__ import annotations

import functools
import math

import numpy as np


def sh_real(l: int, u: np.ndarray) -> np.ndarray:
    """e3nn-convention component-normalised real SH of degree l (l <= 3) of unit vectors u [n, 3]."""
    x, y, z = u[:, 0], u[:, 1], u[:, 2]
    if l == 0:
        return np.ones((u.shape[0], 1))
    if l == 1:
        return math.sqrt(3.0) * np.stack([x, y, z], 1)
    r15, r5 = math.sqrt(15.0), math.sqrt(5.0)
    a0 = r15 * x * z
    a4 = 0.5 * r15 * (z * z - x * x)
    if l == 2:
        return np.stack([a0, r15 * x * y, r5 * (y * y - 0.5 * (x * x + z * z)), r15 * y * z, a4], 1)
    if l == 3:
        q = x * x + z * z
        return np.stack([
            math.sqrt(42.0) / 6.0 * (a0 * z + a4 * x),
            math.sqrt(7.0) * a0 * y,
            math.sqrt(168.0) / 8.0 * (4.0 * y * y - q) * x,
            0.5 * math.sqrt(7.0) * y * (2.0 * y * y - 3.0 * q),
            math.sqrt(168.0) / 8.0 * z * (4.0 * y * y - q),
            math.sqrt(7.0) * a4 * y,
            math.sqrt(42.0) / 6.0 * (a4 * z - a0 * x)], 1)
    raise ValueError(l)


def _sh_complex(l: int, u: np.ndarray) -> np.ndarray:
    from scipy.special import sph_harm_y

    theta = np.arccos(np.clip(u[:, 2], -1.0, 1.0))
    phi = np.arctan2(u[:, 1], u[:, 0])
    return np.stack([sph_harm_y(l, m, theta, phi) for m in range(-l, l + 1)], 1)


@functools.lru_cache(maxsize=None)
def _Q(l: int) -> np.ndarray:
    """Unitary Q with Y_real = Q Y_complex (per point), Y_real normalised to unit integral norm."""
    if l > 3:
        s = 1.0 / math.sqrt(2.0)
        Q = np.zeros((2 * l + 1, 2 * l + 1), dtype=complex)
        for m in range(-l, l + 1):
            a = m + l
            if m < 0:
                Q[a, l + m] = 1j * s
                Q[a, l - m] = -1j * s * (-1) ** m
            elif m == 0:
                Q[a, l] = 1.0
            else:
                Q[a, l - m] = s
                Q[a, l + m] = s * (-1) ** m
        return Q
    rng = np.random.default_rng(99 + l)
    u = rng.normal(size=(200, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    Yr = sh_real(l, u) / math.sqrt(4.0 * math.pi)
    Yc = _sh_complex(l, u)
    Qt, *_ = np.linalg.lstsq(Yc, Yr.astype(complex), rcond=None)
    Q = Qt.T
    assert np.abs(Q @ Q.conj().T - np.eye(2 * l + 1)).max() < 1e-9, "real SH basis not unitary-related"
    return Q


@functools.lru_cache(maxsize=None)
def w3j(l1: int, l2: int, l3: int) -> np.ndarray:
    from sympy.physics.wigner import wigner_3j as sym3j

    cplx = np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1))
    for m1 in range(-l1, l1 + 1):
        for m2 in range(-l2, l2 + 1):
            m3 = -m1 - m2
            if abs(m3) <= l3:
                cplx[m1 + l1, m2 + l2, m3 + l3] = float(sym3j(l1, l2, l3, m1, m2, m3))
    Qi = [np.linalg.inv(_Q(l)) for l in (l1, l2, l3)]
    C = np.einsum("ijk,ia,jb,kc->abc", cplx.astype(complex), Qi[0], Qi[1], Qi[2])
    k = np.unravel_index(np.argmax(np.abs(C)), C.shape)
    C = C / (C[k] / abs(C[k]))                       # remove the global phase
    assert np.abs(C.imag).max() < 1e-9
    C = C.real
    C[np.abs(C) < 1e-13] = 0.0
    C /= np.linalg.norm(C)
    flat = C.reshape(-1)
    nz = np.flatnonzero(np.abs(flat) > 1e-10)
    if flat[nz[0]] < 0:
        C = -C
    return C


# ---------------------------------------------------------------------------------------------- coupling paths
def _par(l):
    return 1 if l % 2 == 0 else -1


SH_IRREPS = [(l, _par(l)) for l in range(4)]


def tp_instructions(node_irreps, target_irreps):
    """'uvu' instructions node_irreps x SH(l<=3) -> target, sorted by output l (stable): [(lo, i1, i2)]."""
    target = set(target_irreps)
    inst = []
    for i1, (l1, p1) in enumerate(node_irreps):
        for i2, (l2, p2) in enumerate(SH_IRREPS):
            for lo in range(abs(l1 - l2), l1 + l2 + 1):
                if (lo, p1 * p2) in target:
                    inst.append((lo, i1, i2))
    return sorted(inst, key=lambda t: t[0])


def _paths(nu, final):
    """Coupling paths of nu copies of 0e+1o+2e+3o, in the recursion order of mace's _wigner_nj, as nested tuples
    (ir_out, tensor [2lo+1, 16^nu])."""
    dims = 16
    offs = [0, 1, 4, 9]
    if nu == 1:
        out = []
        for l in range(4):
            E = np.zeros((2 * l + 1, dims))
            E[:, offs[l]:offs[l] + 2 * l + 1] = np.eye(2 * l + 1)
            out.append(((l, _par(l)), E))
        return out
    ret = []
    for (irl, Cl) in _paths(nu - 1, None):
        ll, pl = irl
        for l in range(4):
            for lo in range(abs(ll - l), ll + l + 1):
                ir = (lo, pl * _par(l))
                if final is not None and ir != final:
                    continue
                W = w3j(lo, ll, l) * math.sqrt(2 * lo + 1)
                T = np.einsum("ajb,jx->axb", W, Cl.reshape(Cl.shape[0], -1))      # [lo, left-flat, l]
                E = np.zeros((2 * lo + 1, Cl.reshape(Cl.shape[0], -1).shape[1], dims))
                E[:, :, offs[l]:offs[l] + 2 * l + 1] = T
                ret.append((ir, E.reshape((2 * lo + 1,) + (dims,) * nu)))
    ret.sort(key=lambda t: (t[0][0], 0 if t[0][1] == _par(t[0][0]) else 1))
    return ret


@functools.lru_cache(maxsize=None)
def U(nu: int, L: int) -> np.ndarray:
    """[2L+1, 16, .., 16, K] coupling tensors of the symmetric contraction (mace U_matrix_real layout + M axis)."""
    target = (L, _par(L))
    Es = [E for (ir, E) in _paths(nu, target) if ir == target]
    return np.stack(Es, -1)
