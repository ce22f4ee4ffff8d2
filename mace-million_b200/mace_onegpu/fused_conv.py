"""Pickle-safe fused convolution module (drop-in for the reference's mace_onegpu.fused_conv.FusedConvTP,
mace_onegpu/fused_conv.py:20-59).

forward(node_feats [n_nodes, nX*128], edge_attrs [E, nY], tp_weights [E, nW*128], edge_index [2, E]) ->
[n_nodes, nO*128]: gather(sender) -> channelwise tensor product -> sum on the receiver, in sm_100a kernels
(torch.ops.mace_b200.conv_tp over mace_b200_conv_tp_fwd / _bwd: receiver- and sender-grouped CSR walks, no atomics),
m_ji never materialised; differentiable w.r.t. node_feats, edge_attrs and tp_weights (the op's registered autograd
formula, torch.ops.mace_b200.conv_tp_backward).  Features use the component-major (ir_mul) layout.  The path table
("segmented polynomial") is the dict of mace_onegpu.o3.channelwise_tp: terms (w, k, m, o, coef) and segment counts.
"""
from __future__ import annotations

import torch

from . import _native as N


class FusedConvTP(torch.nn.Module):
    """gather(sender) -> channel-wise tensor product -> scatter_add(receiver), fused."""

    def __init__(self, segmented_polynomial, weight_numel, irreps_out=None):
        super().__init__()
        tab = segmented_polynomial
        self.m = tab
        self.weight_numel = int(weight_numel)
        self.irreps_out = irreps_out
        self.nX, self.nW, self.nO = int(tab["nX"]), int(tab["nW"]), int(tab["nO"])
        assert self.weight_numel == self.nW * 128, "tp weights must be nW segments of 128 channels"
        self._terms = [(int(w), int(k), int(m), int(o), float(c)) for (w, k, m, o, c) in tab["terms"]]
        self._dev = {}

    def term_tensors(self, device):
        key = str(device)
        if key not in self._dev:
            t = torch.tensor([[w, k, m, o] for (w, k, m, o, _c) in self._terms], dtype=torch.int32, device=device)
            c = torch.tensor([c for (*_x, c) in self._terms], dtype=torch.float32, device=device)
            self._dev[key] = (t.contiguous(), c.contiguous())
        return self._dev[key]

    def __getstate__(self):
        d = self.__dict__.copy()
        d["_dev"] = {}
        return d

    def forward(self, node_feats, edge_attrs, tp_weights, edge_index):
        terms, coef = self.term_tensors(node_feats.device)
        return N.ops().conv_tp(node_feats.float(), edge_attrs.float(), tp_weights.float(), edge_index, terms, coef,
                               self.nO)


def repair_fused_blocks(model):
    """Kept for API compatibility with the reference (fused_conv.py:40-59): the B200 model container has no
    monkeypatched cuEquivariance blocks to repair.  Returns 0."""
    return 0
