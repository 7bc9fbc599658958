"""ZAYA's MoE block on the GPU: ``ZayaModel._moe`` (engine/zaya.py:274-307)
batched over tokens.

Router chain (all f32, one row per token):

    r = W_in h (+ b_in)                       ffn_gate_inp
    r += prev_router * w_eda                  zaya_router_eda (when given)
    state = r                                 returned to the next MoE layer
    r = rmsnorm(r) * norm_w                   ffn_norm
    r = gelu(W_gate r); r = gelu(W_mlp2 r)    ffn_gate, zaya_router_mlp2 (exact GELU)
    logits = W_mlp4 r                         zaya_router_mlp4, E + 1 routes
    p = softmax(logits); e = argmax(p + route_bias); weight = p[e]

Route E is the learned skip route: the token's output is its block input
times p[E].  Otherwise the output is the selected expert's quantised FFN
(``QuantMoE``'s tensor-core path) times p[e].  The linear layers run on the
library's f32 linear kernel (the router kernel), the rest on its element-
and row-wise kernels; nothing falls back to the CPU.
"""
from __future__ import annotations

import torch

from . import _lib
from .moe import QuantMoE, _stream


def _f32(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError('router tensors must be CUDA tensors')
    return t.contiguous().float()


class ZayaRouter:
    def __init__(self, w_in, w_gate, w_mlp2, w_mlp4, norm_w, route_bias, *, b_in=None, b_gate=None, b_mlp2=None,
                 b_mlp4=None, w_eda=None, eps: float = 1e-5):
        self.w = [_f32(w_in), _f32(w_gate), _f32(w_mlp2), _f32(w_mlp4)]
        self.b = [_f32(b_in), _f32(b_gate), _f32(b_mlp2), _f32(b_mlp4)]
        for i in range(1, 4):
            if self.w[i].shape[1] != self.w[i - 1].shape[0]:
                raise ValueError('router layer shapes do not chain')
        self.D, self.R = self.w[0].shape[1], self.w[0].shape[0]
        self.n_routes = self.w[3].shape[0]                 # experts + 1 (skip)
        for w in self.w:
            if w.shape[1] % 4:
                raise ValueError('router input widths must be multiples of 4')
        self.norm_w = _f32(norm_w)
        self.route_bias = _f32(route_bias)
        self.w_eda = _f32(w_eda)
        self.eps = float(eps)
        self.lib = _lib.load()

    def _linear(self, x, i):
        w, b = self.w[i], self.b[i]
        y = torch.empty((x.shape[0], w.shape[0]), dtype=torch.float32, device=x.device)
        _lib.check(self.lib.b200q_moe_router_dev(x.data_ptr(), w.data_ptr(), None if b is None else b.data_ptr(),
                                                 y.data_ptr(), x.shape[0], w.shape[0], w.shape[1], _stream()))
        return y

    def forward(self, h: torch.Tensor, prev_router: torch.Tensor | None = None):
        """(route [T] int32, weight [T] f32, router_state [T, R] f32)."""
        T = h.shape[0]
        r = self._linear(h, 0)
        state = torch.empty_like(r)
        normed = torch.empty_like(r)
        prev = None if prev_router is None or self.w_eda is None else prev_router.contiguous()
        _lib.check(self.lib.b200q_zaya_router_prep_dev(
            r.data_ptr(), None if prev is None else prev.data_ptr(),
            None if prev is None else self.w_eda.data_ptr(), self.norm_w.data_ptr(), T, self.R, self.eps,
            state.data_ptr(), normed.data_ptr(), _stream()))
        a = self._linear(normed, 1)
        _lib.check(self.lib.b200q_gelu_dev(a.data_ptr(), a.numel(), _stream()))
        a = self._linear(a, 2)
        _lib.check(self.lib.b200q_gelu_dev(a.data_ptr(), a.numel(), _stream()))
        logits = self._linear(a, 3)
        ids = torch.empty((T, 1), dtype=torch.int32, device=h.device)
        w = torch.empty((T, 1), dtype=torch.float32, device=h.device)
        _lib.check(self.lib.b200q_moe_topk_dev(logits.data_ptr(), self.route_bias.data_ptr(), T, self.n_routes, 1,
                                               0, ids.data_ptr(), w.data_ptr(), _stream()))
        return ids, w, state

    __call__ = forward


class ZayaMoE:
    """Router chain + top-1 over E experts and the skip route + expert FFN."""

    def __init__(self, router: ZayaRouter, experts: QuantMoE):
        if router.n_routes != experts.E_held + 1 or router.D != experts.D:
            raise ValueError('router must produce experts + 1 routes over d_model inputs')
        self.router, self.experts = router, experts
        self.E = experts.E_held
        self.lib = experts.lib

    def forward(self, h: torch.Tensor, prev_router: torch.Tensor | None = None):
        """(y [T, D] f32, router_state [T, R] f32) for h [T, D] f32."""
        if h.dtype != torch.float32 or not h.is_cuda or h.dim() != 2:
            raise ValueError('h must be a CUDA f32 [T, d_model] tensor')
        h = h.contiguous()
        L = self.experts
        T = h.shape[0]
        ids, w, state = self.router(h, prev_router)
        offsets, slot_of, _, slot_w, xperm = L.dispatch(h, ids, w, n_experts=self.E + 1, k=1)
        out = L.experts(xperm, offsets[:self.E + 1], None)            # routed rows of the E experts
        _lib.check(self.lib.b200q_copy_rows_range_dev(xperm.data_ptr(), out.data_ptr(), offsets.data_ptr(),
                                                      self.E, L.D, xperm.shape[0], _stream()))
        y = L.combine(out, slot_of, T, slot_w, k=1)
        return y, state

    __call__ = forward
