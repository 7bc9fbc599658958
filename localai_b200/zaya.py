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
library's f32 linear kernel (the router kernel) for f32/f16 weights, or on
the quantised GEMV (f32 accumulation) for GGUF block-quantised weights -- the
reference calls ``self._matvec`` on whatever type the checkpoint stores
(engine/zaya.py:279-289, engine/model.py:42-80, which also adds a
``<name>.bias`` tensor when the file has one); the rest runs on the library's
element- and row-wise kernels; nothing falls back to the CPU.
"""
from __future__ import annotations

from typing import NamedTuple

import torch

from . import _lib, ops
from .moe import QuantMoE, _stream

QUANT_TYPES = (2, 8, 12, 13, 14)      # Q4_0, Q8_0, Q4_K, Q5_K, Q6_K


class QuantMatrix(NamedTuple):
    """A [rows, cols] matrix kept as raw GGUF blocks on the device."""
    raw: torch.Tensor                 # CUDA uint8
    ggml_type: int
    rows: int
    cols: int


def _f32(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError('router tensors must be CUDA tensors')
    return t.contiguous().float()


def _weight(w):
    """f32 CUDA tensor, or a QuantMatrix of a supported block type."""
    if isinstance(w, QuantMatrix):
        if w.ggml_type not in QUANT_TYPES:
            raise ValueError(f'router weights of GGML type {w.ggml_type} are not supported')
        if w.raw.dtype != torch.uint8 or not w.raw.is_cuda:
            raise ValueError('QuantMatrix.raw must be a CUDA uint8 tensor')
        ops._check_weights(w.raw, w.ggml_type, w.rows, w.cols)
        return w
    return _f32(w)


def _shape(w):
    return (w.rows, w.cols) if isinstance(w, QuantMatrix) else tuple(w.shape)


class ZayaRouter:
    """Router chain of one ZAYA MoE layer.  Each of ``w_in``, ``w_gate``,
    ``w_mlp2``, ``w_mlp4`` is an f32/f16 CUDA matrix or a ``QuantMatrix``
    (raw GGUF blocks, as a checkpoint stores them); ``from_gguf`` builds the
    router of layer ``layer`` from a ``DeviceGGUF`` by the reference's tensor
    names."""

    def __init__(self, w_in, w_gate, w_mlp2, w_mlp4, norm_w, route_bias, *, b_in=None, b_gate=None, b_mlp2=None,
                 b_mlp4=None, w_eda=None, eps: float = 1e-5):
        self.w = [_weight(w_in), _weight(w_gate), _weight(w_mlp2), _weight(w_mlp4)]
        self.b = [_f32(b_in), _f32(b_gate), _f32(b_mlp2), _f32(b_mlp4)]
        shapes = [_shape(w) for w in self.w]
        for i in range(1, 4):
            if shapes[i][1] != shapes[i - 1][0]:
                raise ValueError('router layer shapes do not chain')
        self.D, self.R = shapes[0][1], shapes[0][0]
        self.n_routes = shapes[3][0]                       # experts + 1 (skip)
        for w, shp in zip(self.w, shapes):
            if not isinstance(w, QuantMatrix) and shp[1] % 4:
                raise ValueError('router input widths must be multiples of 4')
        for b, shp in zip(self.b, shapes):
            if b is not None and b.numel() != shp[0]:
                raise ValueError("router bias length must match its layer's output rows")
        self.norm_w = _f32(norm_w)
        self.route_bias = _f32(route_bias)
        self.w_eda = _f32(w_eda)
        self.eps = float(eps)
        self.lib = _lib.load()

    @classmethod
    def from_gguf(cls, gguf, layer: int, eps: float = 1e-5):
        """Router of MoE layer ``layer`` from a DeviceGGUF, by the names
        engine/zaya.py:278-293 reads (F32/F16 tensors as f32 matrices,
        block-quantised ones kept raw; ``<name>.bias`` added when present)."""
        p = f'blk.{layer}.'

        def mat(name):
            x = gguf.tensors[name]
            if x.ggml_type in QUANT_TYPES:
                rows, cols = x.shape
                return QuantMatrix(gguf.raw(name), x.ggml_type, rows, cols)
            return gguf.tensor_dev(name)

        def vec(name):
            return gguf.tensor_dev(name).reshape(-1) if name in gguf.tensors else None

        def bias(name):
            return vec(name[:-6] + 'bias')

        names = [p + 'ffn_gate_inp.weight', p + 'ffn_gate.weight', p + 'zaya_router_mlp2.weight',
                 p + 'zaya_router_mlp4.weight']
        return cls(*[mat(n) for n in names], vec(p + 'ffn_norm.weight'), vec(p + 'zaya_router_biases.weight'),
                   b_in=bias(names[0]), b_gate=bias(names[1]), b_mlp2=bias(names[2]), b_mlp4=bias(names[3]),
                   w_eda=vec(p + 'zaya_router_eda.weight'), eps=eps)

    def _linear(self, x, i):
        w, b = self.w[i], self.b[i]
        if isinstance(w, QuantMatrix):
            # f32-accurate quantised GEMV (routing decisions need f32, not the bf16 tensor-core path)
            y = ops.gemv(w.raw, x.contiguous(), w.ggml_type, w.rows, w.cols)
            if b is not None:
                y += b
            return y
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

    @classmethod
    def from_gguf(cls, gguf, layer: int, eps: float = 1e-5):
        """MoE block ``layer`` of a DeviceGGUF: the router chain
        (``ZayaRouter.from_gguf``) and the experts' raw tensors
        'blk.<layer>.ffn_gate_up_exps.weight' [E, 2F, D] (gate rows first) and
        'ffn_down_exps.weight' [E, D, F], the ones engine/zaya.py:139-175
        slices one expert at a time (each of its own GGML type).  E, F and D
        come from their shapes; the router must produce E + 1 routes (the last
        one the skip route)."""
        p = f'blk.{layer}.'
        gu, dn = gguf.tensors[p + 'ffn_gate_up_exps.weight'], gguf.tensors[p + 'ffn_down_exps.weight']
        if len(gu.shape) != 3 or len(dn.shape) != 3:
            raise ValueError(f'expert tensors must be [experts, out, in], got {gu.shape} and {dn.shape}')
        E, F2, D = (int(v) for v in gu.shape)
        if F2 % 2 or tuple(int(v) for v in dn.shape) != (E, D, F2 // 2):
            raise ValueError(f'ffn_down_exps shape {dn.shape} does not match ffn_gate_up_exps {gu.shape}')
        router = ZayaRouter.from_gguf(gguf, layer, eps)
        # QuantMoE's own linear router (a placeholder here) is never used: the
        # block routes with the ZAYA chain and calls only its expert stages
        experts = QuantMoE(torch.zeros((E, D), device=gguf.device), gguf.raw(p + 'ffn_gate_up_exps.weight'),
                           gguf.raw(p + 'ffn_down_exps.weight'), d_model=D, d_ff=F2 // 2, top_k=1,
                           renormalize=False, ggml_type=gu.ggml_type, down_type=dn.ggml_type)
        return cls(router, experts)

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
