"""Pickle-safe fused convolution module (drop-in for the reference's mace_onegpu.fused_conv.FusedConvTP,
mace_onegpu/fused_conv.py:20-59).

forward(node_feats [n_nodes, nX*128], edge_attrs [E, nY], tp_weights [E, nW*128], edge_index [2, E]) ->
[n_nodes, nO*128]: gather(sender) -> channelwise tensor product -> scatter-add(receiver) in one sm_100a kernel
(libmace_b200.so: mace_b200_conv_tp_fwd / _bwd), m_ji never materialised; differentiable w.r.t. node_feats,
edge_attrs and tp_weights.  Features use the component-major (ir_mul) layout.  The path table ("segmented
polynomial") is the dict of mace_onegpu.o3.channelwise_tp: terms (w, k, m, o, coef) and segment counts.
"""
from __future__ import annotations

import torch

from . import _native as N


class _ConvTPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X, Y, W, snd, rcv, mod):
        X, Y, W = X.contiguous().float(), Y.contiguous().float(), W.contiguous().float()
        n = X.shape[0]
        out = torch.zeros(n, mod.nO * 128, dtype=torch.float32, device=X.device)
        st = torch.cuda.current_stream(X.device).cuda_stream
        tt, tc = mod.term_tensors(X.device)
        N.check(N.lib().mace_b200_conv_tp_fwd(N.ptr(X), mod.nX, N.ptr(Y), Y.shape[1], N.ptr(W), mod.nW, N.ptr(snd),
                                              N.ptr(rcv), snd.numel(), n, N.ptr(tt), N.ptr(tc), tc.numel(),
                                              N.ptr(out), mod.nO, None, st), "conv_tp_fwd")
        ctx.save_for_backward(X, Y, W, snd, rcv)
        ctx.mod = mod
        return out

    @staticmethod
    def backward(ctx, g):
        X, Y, W, snd, rcv = ctx.saved_tensors
        mod = ctx.mod
        g = g.contiguous().float()
        dX = torch.zeros_like(X) if ctx.needs_input_grad[0] else None
        dY = torch.zeros_like(Y) if ctx.needs_input_grad[1] else None
        dW = torch.zeros_like(W) if ctx.needs_input_grad[2] else None
        st = torch.cuda.current_stream(X.device).cuda_stream
        tt, tc = mod.term_tensors(X.device)
        N.check(N.lib().mace_b200_conv_tp_bwd(N.ptr(X), mod.nX, N.ptr(Y), Y.shape[1], N.ptr(W), mod.nW, N.ptr(snd),
                                              N.ptr(rcv), snd.numel(), X.shape[0], N.ptr(tt), N.ptr(tc), tc.numel(),
                                              N.ptr(g), mod.nO, N.ptr(dX), N.ptr(dY), N.ptr(dW), None, st),
                "conv_tp_bwd")
        return dX, dY, dW, None, None, None


class FusedConvTP(torch.nn.Module):
    """gather(sender) -> channel-wise tensor product -> scatter_add(receiver), fused in one kernel."""

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
        snd = edge_index[0].to(torch.int32).contiguous()
        rcv = edge_index[1].to(torch.int32).contiguous()
        return _ConvTPFn.apply(node_feats, edge_attrs, tp_weights, snd, rcv, self)


def repair_fused_blocks(model):
    """Kept for API compatibility with the reference (fused_conv.py:40-59): the B200 model container has no
    monkeypatched cuEquivariance blocks to repair.  Returns 0."""
    return 0
