"""The library's cell-list neighbour kernels (mace_b200_nbr_count / _fill, mace_b200_verlet_filter) against the host
torch cell list: the same pair set and edge vectors (the GPU orders senders of a receiver by cell scan, the host by
index, so both are compared as sets keyed by (i, j)), for a periodic box, an open set with explicit ghosts, and the
Verlet filter of a skin list at displaced positions."""
import numpy as np
import pytest
import torch

from mace_onegpu import domain as D
from mace_onegpu import neighbors as NB
from mace_onegpu import structures as S

pytestmark = pytest.mark.gpu


def _canon(pi, pj, rij, n):
    pi, pj, rij = pi.long().cpu(), pj.long().cpu(), rij.double().cpu()
    o = torch.argsort(pi * n + pj)
    return pi[o], pj[o], rij[o]


def test_periodic_list_matches_host():
    pos, Z, box = S.water_box(7, seed=3)                  # box 21.7 A: 3 cells of >= 6 A per dimension
    n = len(Z)
    g = NB.neighbor_list(pos, box, 6.0, device="cuda", return_rowptr=True)
    h = NB.neighbor_list(pos, box, 6.0, device="cpu")
    assert torch.all(g[0][1:] >= g[0][:-1])               # receiver-sorted
    assert torch.equal(g[3].cpu(), torch.searchsorted(g[0].long().cpu(), torch.arange(n + 1)))
    a, b = _canon(*g[:3], n), _canon(*h, n)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert float((a[2] - b[2]).abs().max()) < 1e-12
    g2 = NB.neighbor_list(pos, box, 6.0, device="cuda")  # deterministic order
    assert torch.equal(g[1], g2[1]) and torch.equal(g[2], g2[2])


def test_open_list_with_ghosts_matches_host():
    pos, Z, box = S.water_box(8, 4, 4, seed=2)
    dec = D.Decomposition(pos, box, (2, 1, 1), 8.0)
    p, gid, nl = dec.rank_atoms(1)
    g = NB.neighbor_list_open(p, nl, 6.0, device="cuda")
    h = NB.neighbor_list_open(p, nl, 6.0, device="cpu")
    assert int(g[0].max()) < nl and int(g[1].max()) < len(gid)
    a, b = _canon(*g, len(gid)), _canon(*h, len(gid))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert float((a[2] - b[2]).abs().max()) < 1e-12


def test_verlet_filter_matches_direct_list():
    pos, Z, box = S.water_box(8, seed=5)
    n = len(Z)
    x = torch.remainder(torch.as_tensor(pos, device="cuda"), torch.as_tensor(box, device="cuda"))
    vpi, vpj, _, vrow = NB.neighbor_list(x, box, 7.0, device="cuda", return_rowptr=True)
    rng = np.random.default_rng(0)
    x2 = x + torch.as_tensor(rng.uniform(-0.25, 0.25, size=x.shape), device="cuda")   # |move| < skin / 2
    f = NB.verlet_filter(x2, torch.as_tensor(box), vrow, vpj, 6.0)
    d = NB.neighbor_list(x2, box, 6.0, device="cuda")
    a, b = _canon(*f, n), _canon(*d, n)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert float((a[2] - b[2]).abs().max()) < 1e-12
