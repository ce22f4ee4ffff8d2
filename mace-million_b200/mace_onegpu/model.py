"""Two-layer MACE (MACE-MPA-0-medium architecture) parameter container, seeded random initialisation, weights file.

The architecture is the one of mace-torch 0.3.15 ``ScaleShiftMACE`` with ``RealAgnosticDensityInteractionBlock`` as
first and ``RealAgnosticDensityResidualInteractionBlock`` as second interaction (asserted by the reference at
``mace_onegpu/fast_layers.py:117-119``), hidden irreps 128x0e+128x1o, max_ell 3, correlation 3, 8 Bessel functions,
polynomial cutoff p = 5, radial MLP [64, 64, 64] with normalize2mom(SiLU), an 89-element one-hot embedding and a
16-unit SiLU readout MLP on the last layer.  Parameters use the initialisation laws of e3nn / mace-torch
(standard normal weights everywhere; symmetric-contraction weights randn / num_params) drawn from one seeded torch
generator in a fixed order, so a seed defines the model bit for bit.

Parameters are held in float64 (the master copy); the CUDA path folds and casts them (engine.py) and the CPU oracle
uses them as they are.  Feature layout convention used throughout: for irreps with 128 channels per component the
layout is component-major ("ir_mul"): [component][channel].
"""
from __future__ import annotations

import dataclasses
import json
import math

import numpy as np
import torch

from . import o3

FORMAT_VERSION = 1
# element symbols, index = Z (0 = placeholder)
CHEMICAL_SYMBOLS = [
    "X", "H", "He", "Li", "Be", "B", "C", "N", "O", "F", "Ne", "Na", "Mg", "Al", "Si", "P", "S", "Cl", "Ar", "K",
    "Ca", "Sc", "Ti", "V", "Cr", "Mn", "Fe", "Co", "Ni", "Cu", "Zn", "Ga", "Ge", "As", "Se", "Br", "Kr", "Rb", "Sr",
    "Y", "Zr", "Nb", "Mo", "Tc", "Ru", "Rh", "Pd", "Ag", "Cd", "In", "Sn", "Sb", "Te", "I", "Xe", "Cs", "Ba", "La",
    "Ce", "Pr", "Nd", "Pm", "Sm", "Eu", "Gd", "Tb", "Dy", "Ho", "Er", "Tm", "Yb", "Lu", "Hf", "Ta", "W", "Re", "Os",
    "Ir", "Pt", "Au", "Hg", "Tl", "Pb", "Bi", "Po", "At", "Rn", "Fr", "Ra", "Ac",
]


@dataclasses.dataclass
class MACEArch:
    r_max: float = 6.0
    num_bessel: int = 8
    num_poly_cutoff: int = 5
    max_ell: int = 3
    correlation: int = 3
    channels: int = 128
    radial_mlp: tuple = (64, 64, 64)
    readout_mlp: int = 16
    atomic_numbers: tuple = tuple(range(1, 90))
    scale: float = 100.0                 # random-init model: gives O(1 eV/A) forces on the water boxes
    shift: float = 0.0
    seed: int = 0

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self))

    @staticmethod
    def from_dict(d) -> "MACEArch":
        d = dict(d)
        d["radial_mlp"] = tuple(d["radial_mlp"])
        d["atomic_numbers"] = tuple(d["atomic_numbers"])
        return MACEArch(**d)


# ------------------------------------------------------------------------------------------------ derived structure
NODE_IRREPS_L1 = [(0, 1)]                       # 128x0e (embedding, linear_up of layer 1)
HIDDEN_IRREPS = [(0, 1), (1, -1)]               # 128x0e + 128x1o (h1)
TARGET_IRREPS = [(0, 1), (1, -1), (2, 1), (3, -1)]  # 128x{0e,1o,2e,3o} (interaction target / skip irreps)
H2_IRREPS = [(0, 1)]                            # last layer keeps scalars only


def tp_tables():
    """Channelwise TP path tables of the two interaction blocks."""
    return (o3.channelwise_tp(NODE_IRREPS_L1, TARGET_IRREPS), o3.channelwise_tp(HIDDEN_IRREPS, TARGET_IRREPS))


def sc_num_params(L: int, nu: int) -> int:
    return int(o3.sc_U(nu, L).shape[-1])


def silu_normalize2mom_cst() -> float:
    """1 / sqrt(E[silu(z)^2]), z ~ N(0, 1): the normalize2mom constant of e3nn, by Gauss-Hermite quadrature."""
    x, w = np.polynomial.hermite_e.hermegauss(200)
    silu = x / (1.0 + np.exp(-x))
    m2 = float((w * silu * silu).sum() / math.sqrt(2.0 * math.pi))
    return 1.0 / math.sqrt(m2)


# ------------------------------------------------------------------------------------------------ the model
class MACEModel(torch.nn.Module):
    """Parameter container (float64 buffers) of the two-layer MACE, with the attributes the ML-IAP wrapper reads
    (``atomic_numbers``, ``r_max``, ``heads``)."""

    def __init__(self, arch: MACEArch | None = None, state: dict | None = None):
        super().__init__()
        self.arch = arch or MACEArch()
        a = self.arch
        self.atomic_numbers = torch.tensor(a.atomic_numbers, dtype=torch.int64)
        self.r_max = float(a.r_max)
        self.heads = ["default"]
        shapes = self.param_shapes(a)
        if state is None:
            state = self.init_params(a, shapes)
        for name, shp in shapes.items():
            t = torch.as_tensor(state[name], dtype=torch.float64)
            assert tuple(t.shape) == tuple(shp), (name, tuple(t.shape), shp)
            self.register_buffer(name.replace(".", "__"), t.clone())

    # parameter access by dotted name
    def p(self, name: str) -> torch.Tensor:
        return getattr(self, name.replace(".", "__"))

    def params(self) -> dict:
        return {k.replace("__", "."): v for k, v in self.named_buffers() if k != "atomic_numbers"}

    @staticmethod
    def param_shapes(a: MACEArch) -> dict:
        C, Z, nb = a.channels, len(a.atomic_numbers), a.num_bessel
        t1, t2 = tp_tables()
        h = list(a.radial_mlp)
        sh = {}
        sh["node_embedding.weight"] = (Z, C)
        for i, (tab, nup) in enumerate(((t1, 1), (t2, 2))):
            sh[f"interactions.{i}.linear_up.weight"] = (nup, C, C)
            dims = [nb] + h + [tab["nW"] * C]
            for k in range(len(dims) - 1):
                sh[f"interactions.{i}.conv_tp_weights.{k}"] = (dims[k], dims[k + 1])
            sh[f"interactions.{i}.density_fn.weight"] = (nb,)
            sh[f"interactions.{i}.linear.weight"] = (tab["nW"], C, C)
        sh["interactions.0.skip_tp.weight"] = (4, C, Z, C)
        sh["interactions.1.skip_tp.weight"] = (1, C, Z, C)
        for L in (0, 1):
            for nu in range(1, a.correlation + 1):
                sh[f"products.0.sc.{L}.{nu}"] = (Z, sc_num_params(L, nu), C)
        for nu in range(1, a.correlation + 1):
            sh[f"products.1.sc.0.{nu}"] = (Z, sc_num_params(0, nu), C)
        sh["products.0.linear.weight"] = (2, C, C)
        sh["products.1.linear.weight"] = (1, C, C)
        sh["readouts.0.weight"] = (C,)
        sh["readouts.1.linear_1.weight"] = (C, a.readout_mlp)
        sh["readouts.1.linear_2.weight"] = (a.readout_mlp,)
        sh["atomic_energies"] = (Z,)
        return sh

    @staticmethod
    def init_params(a: MACEArch, shapes: dict) -> dict:
        g = torch.Generator().manual_seed(int(a.seed))
        out = {}
        for name, shp in shapes.items():           # dict order = fixed draw order
            if name == "atomic_energies":
                out[name] = torch.zeros(shp, dtype=torch.float64)
                continue
            w = torch.randn(shp, generator=g, dtype=torch.float64)
            if ".sc." in name:
                w = w / shp[1]                      # mace: randn(num_elements, num_params, C) / num_params
            out[name] = w
        return out

    # --------------------------------------------------------------------------------------------- file format
    def save(self, path: str) -> None:
        torch.save({"format": "mace_b200.weights", "version": FORMAT_VERSION, "arch": dataclasses.asdict(self.arch),
                    "state_dict": {k: v.clone() for k, v in self.params().items()}}, path)

    @staticmethod
    def load(path: str) -> "MACEModel":
        d = torch.load(path, map_location="cpu", weights_only=False)
        if d.get("format") != "mace_b200.weights" or int(d.get("version", -1)) != FORMAT_VERSION:
            raise ValueError(f"{path}: not a mace_b200 weights file of version {FORMAT_VERSION}")
        return MACEModel(MACEArch.from_dict(d["arch"]), d["state_dict"])

    def element_symbols(self):
        return [CHEMICAL_SYMBOLS[int(z)] for z in self.arch.atomic_numbers]


def default_model(seed: int = 0, scale: float | None = None) -> MACEModel:
    """The random-init model of the benchmark configurations (seed 0 for water, seed 1 for the alloy)."""
    arch = MACEArch(seed=seed)
    if scale is not None:
        arch.scale = float(scale)
    return MACEModel(arch)
