"""O(3) constants of the MACE architecture, generated from the mathematics (no e3nn / cuEquivariance).

* Real spherical harmonics up to l = 3 in "component" normalisation (sum_m Y_lm(u)^2 = 2l + 1 for |u| = 1),
  written as homogeneous polynomials of the unit vector (the polynomial forms e3nn 0.4 uses).
* Wigner-3j coupling tensors in that real basis, computed as the one-dimensional null space of
  (D_l1 (x) D_l2 (x) D_l3 - I) over random rotations, normalised to unit Frobenius norm with the sign fixed so that
  the first non-zero entry (C order) is positive.
* Channelwise tensor-product path tables: the instruction list of a "uvu" tensor product of node irreps with the SH
  irreps, filtered to the target irreps and sorted by output irrep (the scheme of mace-torch's
  ``tp_out_irreps_with_instructions``), flattened to scalar terms (w, k, m, o, coef) as
  ``mace_onegpu/fused_edge_conv.py:43-68`` (``path_table``) reads them from cuEquivariance.
* Symmetric-contraction coupling tensors U_nu (nu = 1..3) for one output irrep, built by the recursive path
  enumeration of mace-torch's ``U_matrix_real`` / ``_wigner_nj`` (every intermediate coupling kept, component
  normalisation), and their symmetrised monomial form used by the CUDA kernels.

The sign / phase convention of the Wigner-3j tensors is this module's own; parity with e3nn is not pinned (the
library is not available), the rotation- and inversion-invariance tests pin the equivariance.
"""
from __future__ import annotations

import functools
import itertools
import math

import numpy as np

LMAX_SH = 3


# ----------------------------------------------------------------------------------------------- spherical harmonics
def sh_poly(lmax: int, x, y, z):
    """Component-normalised real SH of the unit vector (x, y, z), l = 0..lmax (lmax <= 3), as a list of
    (lmax+1)^2 expressions.  Works on numpy arrays, torch tensors or any type with + - * by constants."""
    assert lmax <= 3
    s3, s5, s15 = math.sqrt(3.0), math.sqrt(5.0), math.sqrt(15.0)
    out = [x * 0 + 1.0]
    if lmax >= 1:
        out += [s3 * x, s3 * y, s3 * z]
    if lmax >= 2:
        y2 = y * y
        x2z2 = x * x + z * z
        s20 = s15 * x * z
        s21 = s15 * x * y
        s22 = s5 * (y2 - 0.5 * x2z2)
        s23 = s15 * y * z
        s24 = 0.5 * s15 * (z * z - x * x)
        out += [s20, s21, s22, s23, s24]
    if lmax >= 3:
        c42, c168, c7 = math.sqrt(42.0) / 6.0, math.sqrt(168.0) / 8.0, math.sqrt(7.0)
        out += [c42 * (s20 * z + s24 * x),
                c7 * s20 * y,
                c168 * (4.0 * y2 - x2z2) * x,
                0.5 * c7 * y * (2.0 * y2 - 3.0 * x2z2),
                c168 * z * (4.0 * y2 - x2z2),
                c7 * s24 * y,
                c42 * (s24 * z - s20 * x)]
    return out


def _sh_generic(l: int, u: np.ndarray) -> np.ndarray:
    """A real orthogonal basis of the degree-l harmonics (component normalisation) for l > 3.  Only used for the
    intermediate irreps of multi-fold couplings, where the basis convention cancels out."""
    from scipy.special import sph_harm_y

    theta = np.arccos(np.clip(u[..., 2], -1.0, 1.0))
    phi = np.arctan2(u[..., 1], u[..., 0])
    cols = []
    for m in range(-l, l + 1):
        Y = sph_harm_y(l, abs(m), theta, phi)
        if m < 0:
            v = math.sqrt(2.0) * Y.imag
        elif m == 0:
            v = Y.real
        else:
            v = math.sqrt(2.0) * Y.real
        cols.append(v * math.sqrt(4.0 * math.pi))
    return np.stack(cols, axis=-1)


def sh_np(lmax: int, v: np.ndarray) -> np.ndarray:
    """SH of the direction of v [..., 3] (normalised internally), fp64 numpy, l = 0..lmax (lmax <= 3)."""
    v = np.asarray(v, dtype=np.float64)
    u = v / np.linalg.norm(v, axis=-1, keepdims=True)
    comps = sh_poly(lmax, u[..., 0], u[..., 1], u[..., 2])
    return np.stack([np.broadcast_to(c, u.shape[:-1]) for c in comps], axis=-1)


def sh_block(l: int, u: np.ndarray) -> np.ndarray:
    """Degree-l block [.., 2l+1] of the real SH of unit vectors u (any l; the e3nn polynomial basis for l <= 3)."""
    if l <= LMAX_SH:
        return sh_np(l, u)[..., l * l:(l + 1) ** 2]
    return _sh_generic(l, u)


# ----------------------------------------------------------------------------------------------- rotations, Wigner D
def _random_rotation(rng: np.random.Generator) -> np.ndarray:
    q, r = np.linalg.qr(rng.normal(size=(3, 3)))
    q = q * np.sign(np.diag(r))
    if np.linalg.det(q) < 0:
        q[:, 0] = -q[:, 0]
    return q


def wigner_D(l: int, R: np.ndarray) -> np.ndarray:
    """Representation matrix of rotation R on the degree-l real SH: Y_l(R u) = D Y_l(u)."""
    if l == 0:
        return np.ones((1, 1))
    rng = np.random.default_rng(12345 + l)
    u = rng.normal(size=(64, 3))
    u = u / np.linalg.norm(u, axis=-1, keepdims=True)
    Y = sh_block(l, u)
    Yr = sh_block(l, u @ R.T)
    Dt, *_ = np.linalg.lstsq(Y, Yr, rcond=None)
    return Dt.T


@functools.lru_cache(maxsize=None)
def wigner_3j(l1: int, l2: int, l3: int) -> np.ndarray:
    """Invariant coupling tensor C[m1, m2, m3] of the real SH basis, ||C|| = 1, first non-zero entry positive."""
    if not (abs(l1 - l2) <= l3 <= l1 + l2):
        raise ValueError(f"triangle violated: {l1} {l2} {l3}")
    rng = np.random.default_rng(7 + 100 * l1 + 10 * l2 + l3)
    d = (2 * l1 + 1) * (2 * l2 + 1) * (2 * l3 + 1)
    rows = []
    for _ in range(3):
        R = _random_rotation(rng)
        K = np.kron(np.kron(wigner_D(l1, R), wigner_D(l2, R)), wigner_D(l3, R))
        rows.append(K - np.eye(d))
    A = np.concatenate(rows, 0)
    _, s, vt = np.linalg.svd(A)
    if s[-1] > 1e-9 or (d > 1 and s[-2] < 1e-6):
        raise RuntimeError(f"w3j({l1},{l2},{l3}): null space is not one-dimensional (s={s[-2:]})")
    c = vt[-1].copy()
    c[np.abs(c) < 1e-12] = 0.0
    c /= np.linalg.norm(c)
    nz = np.flatnonzero(np.abs(c) > 1e-10)
    if c[nz[0]] < 0:
        c = -c
    return c.reshape(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1)


# ----------------------------------------------------------------------------------------------- irreps helpers
def natural_parity(l: int) -> int:
    return 1 if l % 2 == 0 else -1


def irrep_sort_key(ir):
    """e3nn ordering of irreps: by l, natural parity first."""
    l, p = ir
    return (l, 0 if p == natural_parity(l) else 1)


def irreps_dim(irs) -> int:
    return sum(2 * l + 1 for (l, _p) in irs)


def sh_irreps(lmax: int = LMAX_SH):
    return [(l, natural_parity(l)) for l in range(lmax + 1)]


# ----------------------------------------------------------------------------------------------- channelwise TP
def channelwise_tp(node_irreps, target_irreps, lmax: int = LMAX_SH):
    """Instruction table of the 'uvu' channelwise tensor product node_irreps (x) SH(lmax) -> mid irreps.

    Returns dict(mid=[(l, p, i1, i2)], terms=[(w, k, m, o, coef)], nW, nX, nY, nO, lin_groups) where
      w = mid entry (= TP weight segment), k = node component, m = SH component, o = mid component, and
      coef = sqrt(2 l_out + 1) * w3j(l1, l2, l_out)[m1, m2, m_out] (component normalisation, one path per output
      entry, so the element path normalisation is 1).
    lin_groups[l] = list of mid entries with output l (consumed by the following per-l linear)."""
    shi = sh_irreps(lmax)
    target = set(target_irreps)
    inst = []
    for i1, (l1, p1) in enumerate(node_irreps):
        for i2, (l2, p2) in enumerate(shi):
            for lo in range(abs(l1 - l2), l1 + l2 + 1):
                if (lo, p1 * p2) in target:
                    inst.append((lo, p1 * p2, i1, i2))
    order = sorted(range(len(inst)), key=lambda k: irrep_sort_key(inst[k][:2]))
    mid = [inst[k] for k in order]
    xoff = np.cumsum([0] + [2 * l + 1 for (l, _p) in node_irreps]).tolist()
    terms = []
    ooff = 0
    lin_groups = {}
    for w, (lo, po, i1, i2) in enumerate(mid):
        l1 = node_irreps[i1][0]
        l2 = shi[i2][0]
        C = wigner_3j(l1, l2, lo) * math.sqrt(2 * lo + 1)
        for m1 in range(2 * l1 + 1):
            for m2 in range(2 * l2 + 1):
                for mo in range(2 * lo + 1):
                    v = float(C[m1, m2, mo])
                    if abs(v) > 1e-12:
                        terms.append((w, xoff[i1] + m1, l2 * l2 + m2, ooff + mo, v))
        lin_groups.setdefault(lo, []).append(w)
        ooff += 2 * lo + 1
    return dict(mid=mid, terms=terms, nW=len(mid), nX=xoff[-1], nY=(lmax + 1) ** 2, nO=ooff, lin_groups=lin_groups)


def mid_offsets(tab):
    """Component offset of every mid entry (its output segment start)."""
    offs, o = [], 0
    for (lo, _p, _i1, _i2) in tab["mid"]:
        offs.append(o)
        o += 2 * lo + 1
    return offs


# ----------------------------------------------------------------------------------------------- symmetric contraction
def _wigner_nj(irreps_list, final=None):
    """All coupling paths of len(irreps_list) inputs (each a list of (l, p), multiplicity 1) to an output irrep.
    Returns [((l, p), E)] with E [2l+1, d_1, ..., d_n] (component normalisation), sorted by output irrep.
    ``final`` restricts the last coupling to one output irrep (the intermediate couplings are all kept)."""
    if len(irreps_list) == 1:
        (irs,) = irreps_list
        d = irreps_dim(irs)
        eye = np.eye(d)
        ret, i = [], 0
        for (l, p) in irs:
            ret.append(((l, p), eye[i:i + 2 * l + 1]))
            i += 2 * l + 1
        return ret
    left_list, right = irreps_list[:-1], irreps_list[-1]
    dims_left = [irreps_dim(x) for x in left_list]
    d_right = irreps_dim(right)
    ret = []
    for (ir_l, C_left) in _wigner_nj(left_list):
        ll, pl = ir_l
        i = 0
        for (l, p) in right:
            for lo in range(abs(ll - l), ll + l + 1):
                if final is not None and (lo, pl * p) != final:
                    continue
                C = wigner_3j(lo, ll, l) * math.sqrt(2 * lo + 1)             # [out, left, right]
                C = np.einsum("jk,ijl->ikl", C_left.reshape(C_left.shape[0], -1), C)
                C = C.reshape(2 * lo + 1, *dims_left, 2 * l + 1)
                E = np.zeros((2 * lo + 1, *dims_left, d_right))
                E[..., i:i + 2 * l + 1] = C
                ret.append(((lo, pl * p), E))
            i += 2 * l + 1
    order = sorted(range(len(ret)), key=lambda k: irrep_sort_key(ret[k][0]))
    return [ret[k] for k in order]


@functools.lru_cache(maxsize=None)
def sc_U(nu: int, L: int, lmax: int = LMAX_SH) -> np.ndarray:
    """U_nu for output irrep (L, natural parity): [2L+1, 16, ..., 16 (nu times), K] (K = number of coupling paths)."""
    irs = sh_irreps(lmax)
    target = (L, natural_parity(L))
    Es = [E for (ir, E) in _wigner_nj([irs] * nu, final=target) if ir == target]
    if not Es:
        d = irreps_dim(irs)
        return np.zeros((2 * L + 1,) + (d,) * nu + (0,))
    return np.stack(Es, axis=-1)


def monomials(nu: int, d: int = 16):
    return list(itertools.combinations_with_replacement(range(d), nu))


@functools.lru_cache(maxsize=None)
def sc_monomial_form(nu: int, L: int, lmax: int = LMAX_SH):
    """Symmetrised U_nu in the monomial basis: (monos [(i1<=..<=inu)], Usym [2L+1, n_mono, K]) keeping only
    monomials with a non-zero coefficient.  poly_M(x) = sum_mono sum_k Usym[M, mono, k] w_k prod x_i."""
    U = sc_U(nu, L, lmax)
    K = U.shape[-1]
    d = U.shape[1]
    rows, keep = [], []
    for mono in monomials(nu, d):
        acc = np.zeros((2 * L + 1, K))
        for perm in set(itertools.permutations(mono)):
            acc += U[(slice(None),) + perm]
        if np.abs(acc).max() > 1e-12:
            keep.append(mono)
            rows.append(acc)
    if not keep:
        return [], np.zeros((2 * L + 1, 0, K))
    return keep, np.stack(rows, axis=1)


# ----------------------------------------------------------------------------------------------- coefficient layout
def sc_entries(Ls, lmax: int = LMAX_SH, correlation: int = 3):
    """Canonical order of the per-(species, channel) coefficients of a symmetric contraction with outputs Ls:
    for L in Ls, nu = 1..correlation, monomial (sorted indices, combinations order), output component M.
    Returns [(L, M, nu, mono, row)] where row [K_{L,nu}] maps the contraction weights w[k] to the coefficient."""
    out = []
    for L in Ls:
        for nu in range(1, correlation + 1):
            monos, Us = sc_monomial_form(nu, L, lmax)
            for a, mono in enumerate(monos):
                for M in range(2 * L + 1):
                    row = Us[M, a]
                    if np.abs(row).max() > 1e-12:
                        out.append((L, M, nu, tuple(mono), row))
    return out


def sc_fingerprint(entries) -> int:
    """FNV-1a 64-bit hash of the entry order (L, M, nu, mono) shared by the host folding and the generated kernels."""
    h = 0xCBF29CE484222325
    for (L, M, nu, mono, _row) in entries:
        for v in (L, M, nu, *mono, 255):
            h ^= int(v) & 0xFF
            h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h
