"""TEST INFRASTRUCTURE: run the reference's own Python code for this path on the CPU, with the oracle's block math.

The reference's driver code (ShiQiaoL/mace-million, ``mace_onegpu/``) needs only torch: the ML-IAP entry point
``mliap_threepass.py:155-616`` (ThreePassMLIAP.compute_forces), the three-pass evaluator
``receiver_chunk_mace.py:82-388`` (Morton-ordered System, LocalGraph chunk topology with padding, ReceiverChunkMACE),
the receiver-only layer order ``fast_layers.py:20-223`` (FastLayers, SpeciesSkip), the exact density-projection
layer 1 ``ace_layer1.py:23-105`` (ACELayer1), the exchange column split ``mliap_threepass.py:40-55`` and the spline
tables ``conv_spline.py:230-249`` / ``spline_radial.py:37-151``.  What it calls into is mace-torch / e3nn / cuEquivariance
(absent here): the model's blocks.  ``OracleMACE`` gives the reference that model interface (the attribute names and
call signatures of mace-torch 0.3.15's ScaleShiftMACE with RealAgnosticDensity(Residual)InteractionBlock), each block
evaluated by ``oracle.mace_ref.MaceRef`` in fp64.  Running the reference's code on it pins the oracle's three-pass
driver, layer order, ML-IAP semantics and spline tables against the reference itself; the block math stays the
oracle's restatement of mace-torch / e3nn.

``reference_env(path)`` imports the reference package under a private name (``_mace_ref_pkg``, so that it does not
collide with this repository's ``mace_onegpu``) with three stand-ins for what this container lacks, active only
inside the ``with`` block: ``ase.data.chemical_symbols`` (read by ThreePassMLIAP.__init__), ``e3nn.o3.Irreps(s).dim``
(read by FastLayers.__init__ for the skip widths) and a no-op ``torch.cuda.synchronize`` (the reference synchronises
between passes; there is no CUDA device here).  Bytecode writing is off inside the block, so that importing leaves
the reference checkout untouched.

Layouts inside the adapter: the tensor product's output (the "mid" features between conv_tp and linear) is
cuEquivariance's "ir_mul" order, per irrep a [component][channel] block (index o * C + c), which the reference's
ACELayer1 writes itself (its 'seg' layout); the other flat features are "mul_ir", per irrep a [channel][component]
block (index c * (2l + 1) + m); h1 rows are the oracle's [C, 4] (0e | 1o) flattened, which only the adapter's own
blocks read (the reference stores H1 rows without looking inside).  The radial MLP is a sequence of layer modules
with the attributes of e3nn's FullyConnectedNet layers that ACELayer1 reads (h_in, weight, act, var_in, var_out).
"""
from __future__ import annotations

import contextlib
import importlib.util
import math
import os
import re
import sys
import types

import torch

from oracle import mace_ref

PKG = "_mace_ref_pkg"


# ---------------------------------------------------------------------------------------------- the reference package
def _fake_e3nn():
    e3nn = types.ModuleType("e3nn")
    o3 = types.ModuleType("e3nn.o3")

    class Irreps:
        """dim of an irreps string such as '128x0e+128x1o' (sum of mul * (2l + 1))."""

        def __init__(self, s):
            self.dim = sum(int(mul) * (2 * int(l) + 1) for mul, l in re.findall(r"(\d+)x(\d+)[eo]", str(s)))

    o3.Irreps = Irreps
    e3nn.o3 = o3
    return {"e3nn": e3nn, "e3nn.o3": o3}


def _fake_ase():
    from mace_onegpu.model import CHEMICAL_SYMBOLS

    ase = types.ModuleType("ase")
    data = types.ModuleType("ase.data")
    data.chemical_symbols = list(CHEMICAL_SYMBOLS)
    ase.data = data
    return {"ase": ase, "ase.data": data}


def _load_package(ref_root):
    """The reference's mace_onegpu package as module PKG (its relative imports resolve inside it)."""
    if PKG in sys.modules:
        return sys.modules[PKG]
    pdir = os.path.join(ref_root, "mace_onegpu")
    spec = importlib.util.spec_from_file_location(PKG, os.path.join(pdir, "__init__.py"),
                                                  submodule_search_locations=[pdir])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules[PKG] = pkg
    spec.loader.exec_module(pkg)
    return pkg


@contextlib.contextmanager
def reference_env(ref_root):
    """Yields a loader ``mod(name)`` of the reference's modules; stand-ins active inside the block only."""
    stand_ins = {}
    for name, mod in {**_fake_e3nn(), **_fake_ase()}.items():
        if name not in sys.modules:
            stand_ins[name] = mod
    sync, nobytecode = torch.cuda.synchronize, sys.dont_write_bytecode
    sys.modules.update(stand_ins)
    torch.cuda.synchronize = lambda *a, **k: None
    sys.dont_write_bytecode = True              # the reference checkout is read-only: no __pycache__ there
    try:
        _load_package(ref_root)

        def mod(name):
            return importlib.import_module(f"{PKG}.{name}")

        yield mod
    finally:
        torch.cuda.synchronize, sys.dont_write_bytecode = sync, nobytecode
        for name in stand_ins:
            sys.modules.pop(name, None)


# ---------------------------------------------------------------------------------------------- flat layouts
def _flat(parts):
    """list of [n, C, 2l+1] -> [n, sum C (2l+1)] in mul_ir order."""
    return torch.cat([p.reshape(p.shape[0], -1) for p in parts], -1)


def _unflat(x, ls, C):
    """inverse of _flat for the irreps ls."""
    out, o = [], 0
    for l in ls:
        w = C * (2 * l + 1)
        out.append(x[:, o:o + w].reshape(x.shape[0], C, 2 * l + 1))
        o += w
    assert o == x.shape[1], (o, x.shape)
    return out


def _flat_ir(parts):
    """list of [n, C, 2l+1] -> [n, sum (2l+1) C] in ir_mul order (index o * C + c)."""
    return torch.cat([p.transpose(1, 2).reshape(p.shape[0], -1) for p in parts], -1)


def _unflat_ir(x, ls, C):
    """inverse of _flat_ir for the irreps ls."""
    out, o = [], 0
    for l in ls:
        w = C * (2 * l + 1)
        out.append(x[:, o:o + w].reshape(x.shape[0], 2 * l + 1, C).transpose(1, 2))
        o += w
    assert o == x.shape[1], (o, x.shape)
    return out


def _species(node_attrs):
    """Column of each one-hot row (the reference builds node_attrs with one_hot; the blocks here need one-hot)."""
    s = node_attrs.argmax(1)
    assert bool((node_attrs.sum(1) == 1).all()) and bool((node_attrs.max(1).values == 1).all()), "one-hot node_attrs"
    return s


def _per_species(x, spec, fn):
    """out[rows of species z] = fn(x[rows], z), rows grouped by species (fn linear in its input)."""
    out = None
    for z in torch.unique(spec).tolist():
        sel = (spec == z).nonzero().flatten()
        y = fn(x[sel], z)
        if out is None:
            out = torch.zeros((x.shape[0],) + tuple(y.shape[1:]), dtype=y.dtype)
        out = out.index_put((sel,), y)
    return out


# ---------------------------------------------------------------------------------------------- the blocks
class _Fn(torch.nn.Module):
    """A parameter-free module around a function of the oracle (deep-copyable, .double()-able)."""

    def __init__(self, fn):
        super().__init__()
        self.fn = fn

    def forward(self, *args):
        return self.fn(*args)


class _FCLayer(torch.nn.Module):
    """One layer of the bias-free radial MLP, y = act * silu(h W / sqrt(h_in)) (act = the normalize2mom constant) or,
    for the last layer (act None), y = h W / sqrt(h_in): the oracle's radial_mlp step by step."""

    def __init__(self, W, act):
        super().__init__()
        self.register_buffer("weight", W)
        self.h_in, self.act, self.var_in, self.var_out = int(W.shape[0]), act, 1, 1

    def forward(self, h):
        z = h @ self.weight / math.sqrt(self.h_in)
        return z if self.act is None else self.act * torch.nn.functional.silu(z)


class _Interaction(torch.nn.Module):
    def __init__(self, ref: mace_ref.MaceRef, i: int):
        super().__init__()
        self.ref, self.i, C = ref, i, ref.C
        self.mid_ls = [lo for (lo, _a, _b) in ref.inst[i]]
        P = ref.P
        if i == 0:
            self.irreps_out = f"{C}x0e+{C}x1o+{C}x2e+{C}x3o"
            self.linear_up = _Fn(lambda x: x @ P["interactions.0.linear_up.weight"][0] / math.sqrt(C))
        else:
            self.node_feats_irreps = f"{C}x0e+{C}x1o"

            def up(x):
                h = x.reshape(x.shape[0], C, 4)
                Wu = P["interactions.1.linear_up.weight"]
                return torch.cat([torch.einsum("ncm,cd->ndm", h[:, :, 0:1], Wu[0]),
                                  torch.einsum("ncm,cd->ndm", h[:, :, 1:4], Wu[1])], -1).reshape(x.shape[0], -1) \
                    / math.sqrt(C)

            self.linear_up = _Fn(up)
        nl = 0
        while f"interactions.{i}.conv_tp_weights.{nl + 1}" in P:
            nl += 1
        self.conv_tp_weights = torch.nn.Sequential(
            *[_FCLayer(P[f"interactions.{i}.conv_tp_weights.{k}"], ref.cst if k < nl else None) for k in range(nl + 1)])
        w = P[f"interactions.{i}.density_fn.weight"]
        self.density_fn = _Fn(lambda feats: feats @ w.unsqueeze(-1) / math.sqrt(w.shape[0]))
        self.conv_tp = _Fn(self._conv)
        self.linear = _Fn(lambda msg: _flat(ref.linear_mid(i, _unflat_ir(msg, self.mid_ls, C))))
        self.skip_tp = _Fn(self._skip)
        self.reshape = _Fn(lambda x: torch.cat(_unflat(x, [0, 1, 2, 3], C), -1))

    def _conv(self, node_feats, edge_attrs, tp_weights, edge_index):
        """gather(sender) -> channelwise TP -> scatter_add(receiver) over all rows of node_feats (FusedConvTP)."""
        C, n = self.ref.C, node_feats.shape[0]
        if self.i == 0:
            X = [node_feats.reshape(n, C, 1)]
        else:
            v = node_feats.reshape(n, C, 4)
            X = [v[:, :, 0:1], v[:, :, 1:4]]
        mid = self.ref.conv(self.i, X, edge_attrs, tp_weights, edge_index[0].long(), edge_index[1].long(), n)
        return _flat_ir(mid)

    def _skip(self, x, node_attrs):
        """FullyConnectedTensorProduct(x, one-hot species): per-species channel mixing, 1/sqrt(C Z)."""
        ref, C, Z = self.ref, self.ref.C, self.ref.Z
        spec = _species(node_attrs)
        if self.i == 0:
            Ws = ref.P["interactions.0.skip_tp.weight"]                                    # [4, C, Z, C]
            parts = _unflat(x, [0, 1, 2, 3], C)
            return _flat([_per_species(p, spec, lambda xs, z, l=l: torch.einsum("ncm,cd->ndm", xs, Ws[l][:, z, :]))
                          / math.sqrt(C * Z) for l, p in enumerate(parts)])
        Wsk = ref.P["interactions.1.skip_tp.weight"][0]                                    # [C, Z, C]
        h0 = x.reshape(x.shape[0], C, 4)[:, :, 0]
        return _per_species(h0, spec, lambda xs, z: xs @ Wsk[:, z, :]) / math.sqrt(C * Z)


class RealAgnosticDensityInteractionBlock(_Interaction):
    """Layer-1 interaction (the class name FastLayers asserts, fast_layers.py:117-118)."""

    def __init__(self, ref):
        super().__init__(ref, 0)


class RealAgnosticDensityResidualInteractionBlock(_Interaction):
    """Layer-2 interaction (the class name FastLayers asserts, fast_layers.py:117-119)."""

    def __init__(self, ref):
        super().__init__(ref, 1)


class _Product(torch.nn.Module):
    """EquivariantProductBasisBlock: symmetric contraction (correlation 3) + linear (+ sc on the last layer)."""

    def __init__(self, ref, k):
        super().__init__()
        self.ref, self.k = ref, k

    def forward(self, node_feats, sc, node_attrs):
        ref, C = self.ref, self.ref.C
        spec = _species(node_attrs)
        if self.k == 0:
            Wp = ref.P["products.0.linear.weight"]
            A0 = ref.sym_contract("products.0", 0, node_feats, spec)
            A1 = ref.sym_contract("products.0", 1, node_feats, spec)
            h = torch.cat([torch.einsum("ncm,cd->ndm", A0, Wp[0]), torch.einsum("ncm,cd->ndm", A1, Wp[1])], -1)
            h = (h / math.sqrt(C)).reshape(h.shape[0], -1)
        else:
            A = ref.sym_contract("products.1", 0, node_feats, spec)[:, :, 0]
            h = A @ ref.P["products.1.linear.weight"][0] / math.sqrt(C)
        return h if sc is None else h + sc


class _Readout(torch.nn.Module):
    def __init__(self, ref, k):
        super().__init__()
        self.ref, self.k = ref, k

    def forward(self, h, heads=None):
        ref, C = self.ref, self.ref.C
        if self.k == 0:
            return ref.readout1(h.reshape(h.shape[0], C, 4)).reshape(-1, 1)
        z = h @ ref.P["readouts.1.linear_1.weight"] / math.sqrt(C)
        a = ref.cst * torch.nn.functional.silu(z)
        w2 = ref.P["readouts.1.linear_2.weight"]
        return (a @ w2 / math.sqrt(w2.shape[0])).reshape(-1, 1)


class OracleMACE(torch.nn.Module):
    """The two-layer MACE with mace-torch's module interface, every block evaluated by the oracle (fp64)."""

    def __init__(self, ref: mace_ref.MaceRef, atomic_numbers):
        super().__init__()
        self.ref = ref
        self.register_buffer("atomic_numbers", torch.as_tensor(list(atomic_numbers), dtype=torch.int64))
        self.r_max = ref.rmax
        self.heads = ["default"]
        self.probe = torch.nn.Parameter(torch.zeros(1, dtype=torch.float64), requires_grad=False)   # dtype / device
        self.spherical_harmonics = _Fn(mace_ref.sh_torch)
        self.radial_embedding = _Fn(lambda lengths, node_attrs, edge_index, zs: (ref.bessel_cut(lengths), None))
        self.node_embedding = _Fn(lambda na: na @ ref.P["node_embedding.weight"] / math.sqrt(ref.Z))
        self.interactions = torch.nn.ModuleList([RealAgnosticDensityInteractionBlock(ref),
                                                 RealAgnosticDensityResidualInteractionBlock(ref)])
        self.products = torch.nn.ModuleList([_Product(ref, 0), _Product(ref, 1)])
        self.readouts = torch.nn.ModuleList([_Readout(ref, 0), _Readout(ref, 1)])

    def scale_shift(self, x, heads):
        return self.ref.scale * x + self.ref.shift

    def atomic_energies_fn(self, node_attrs):
        return (node_attrs @ self.ref.P["atomic_energies"]).reshape(-1, 1)
