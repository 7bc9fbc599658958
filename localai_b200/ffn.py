"""Dense quantised FFN of the reference decoder on the GPU.

``engine/model.py:161-166`` (and :230-233 for decode) computes, per layer,

    gate = W_gate x;  up = W_up x;  y = W_down (silu(gate) * up)

with three ``GGUFFile.matvec/matmul`` calls on the raw GGUF tensors
(``ffn_gate``/``ffn_up`` [F, D], ``ffn_down`` [D, F]).  ``QuantFFN`` keeps the
three tensors on the device (gate and up concatenated once into [2F, D]) and
runs, for T tokens:

* T <= ``gemv_max_tokens``: one GEMV over [gate; up] (f32 accumulation,
  weights streamed once per call), ``b200q_silu_mul_dev``, one GEMV over down
  -- the decode path, HBM-bound;
* larger T: the tensor-core GEMM in gate/up mode (fused SiLU * up, bf16
  activations) and in plain mode for down -- the prefill path.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .moe import _stream

SUPPORTED_GEMV = (2, 8, 12, 13, 14)
SUPPORTED_GEMM = (2, 8, 12, 13, 14)


class QuantFFN:
    def __init__(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, *, d_model: int, d_ff: int,
                 ggml_type: int = 12, down_type: int | None = None, gemv_max_tokens: int = 16):
        self.D, self.F = d_model, d_ff
        self.t_gu = ggml_type
        self.t_dn = ggml_type if down_type is None else down_type
        if self.t_gu not in SUPPORTED_GEMV or self.t_dn not in SUPPORTED_GEMV:
            raise NotImplementedError(f'unsupported GGML types {self.t_gu}/{self.t_dn}')
        for name, t, rows, cols in (('gate', gate, d_ff, d_model), ('up', up, d_ff, d_model),
                                    ('down', down, d_model, d_ff)):
            if t.dtype != torch.uint8 or not t.is_cuda:
                raise ValueError(f'{name} must be a CUDA uint8 tensor of raw GGUF blocks')
        self.gate_up = torch.cat([gate.reshape(-1), up.reshape(-1)])
        self.down = down.contiguous().reshape(-1)
        ops._check_weights(self.gate_up, self.t_gu, 2 * d_ff, d_model)
        ops._check_weights(self.down, self.t_dn, d_model, d_ff)
        self.gemv_max_tokens = gemv_max_tokens
        self._gemm_w = None
        self._row_off = {}             # T -> int32 [0, T] on the device (kept, so calls can be graph-captured)
        self.lib = _lib.load()

    def _gemm_weights(self):
        """16-byte-row copies for the tensor-core path (made once, if needed)."""
        if self._gemm_w is None:
            if self.t_gu not in SUPPORTED_GEMM or self.t_dn not in SUPPORTED_GEMM:
                raise NotImplementedError('the tensor-core path supports Q4_0, Q8_0, Q4_K, Q5_K and Q6_K')
            gu, s_gu = ops.pad_rows(self.gate_up, 2 * self.F, ops.packed_row_bytes(self.t_gu, self.D))
            dn, s_dn = ops.pad_rows(self.down, self.D, ops.packed_row_bytes(self.t_dn, self.F))
            self._gemm_w = (gu, s_gu, dn, s_dn)
        return self._gemm_w

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """y [T, D] (f32) for x [T, D] or [D] (f32, CUDA)."""
        squeeze = x.dim() == 1
        x2 = (x.reshape(1, -1) if squeeze else x).contiguous()
        if x2.dtype != torch.float32 or not x2.is_cuda or x2.shape[1] != self.D:
            raise ValueError('x must be a CUDA f32 [T, d_model] tensor')
        T, dev = x2.shape[0], x2.device
        use_gemm = T > self.gemv_max_tokens and self.t_gu in SUPPORTED_GEMM and self.t_dn in SUPPORTED_GEMM \
            and self.F % 64 == 0 and self.D % 128 == 0
        if not use_gemm:
            gu = ops.gemv(self.gate_up, x2, self.t_gu, 2 * self.F, self.D)
            act = torch.empty((T, self.F), dtype=torch.float32, device=dev)
            _lib.check(self.lib.b200q_silu_mul_dev(gu.data_ptr(), T, self.F, act.data_ptr(), self.F, _stream()))
            y = ops.gemv(self.down, act, self.t_dn, self.D, self.F)
        else:
            gu_w, s_gu, dn_w, s_dn = self._gemm_weights()
            off = self._row_off.get(T)
            if off is None:
                off = self._row_off[T] = torch.tensor([0, T], dtype=torch.int32, device=dev)
            xb = x2.to(torch.bfloat16)
            act = ops.gemm_quant(xb, gu_w, off, k=self.D, n_feat=self.F, w_rows_per_group=2 * self.F,
                                 up_offset=self.F, ggml_type=self.t_gu, w_row_bytes=s_gu)
            y = ops.gemm_quant(act, dn_w, off, k=self.F, n_feat=self.D, w_rows_per_group=self.D,
                               ggml_type=self.t_dn, w_row_bytes=s_dn, out_dtype=torch.float32)
        return y.reshape(self.D) if squeeze else y

    __call__ = forward
