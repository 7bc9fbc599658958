"""PyTorch-facing device operations over libb200quant (device-pointer C ABI).

Tensors stay on the GPU; work is enqueued on the current torch stream.  Weight
tensors are raw GGUF block bytes (``torch.uint8``) of a [rows, cols] matrix.
"""
from __future__ import annotations

import torch

from . import _lib

BLOCK = {2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
# unquantised GGML types the GEMV also takes: bytes per value (F32, F16)
DENSE = {0: 4, 1: 2}


def _stream():
    return torch.cuda.current_stream().cuda_stream


def row_bytes(ggml_type: int, cols: int) -> int:
    if ggml_type in DENSE:
        return cols * DENSE[ggml_type]
    vals, nbytes = BLOCK[ggml_type]
    if cols % vals:
        raise ValueError(f'cols={cols} not a multiple of block {vals}')
    return (cols // vals) * nbytes


def _check_weights(w: torch.Tensor, ggml_type: int, rows: int, cols: int):
    if ggml_type not in BLOCK and ggml_type not in DENSE:
        raise ValueError(f'unsupported GGML type {ggml_type}')
    if not w.is_cuda or w.dtype != torch.uint8:
        raise ValueError('weights must be a CUDA uint8 tensor of raw GGUF blocks')
    if w.numel() < rows * row_bytes(ggml_type, cols):
        raise ValueError('weight tensor smaller than rows * row_bytes')


def dequantize(w: torch.Tensor, ggml_type: int, shape, dtype=torch.float32) -> torch.Tensor:
    """Exact f32 (or bf16-rounded) dequantization (engine/dequant.py:27-167)."""
    vals, nbytes = BLOCK[ggml_type]
    n = 1
    for s in shape:
        n *= int(s)
    if n % vals:
        raise ValueError(f'{n} elements is not divisible by block size {vals}')
    nblocks = n // vals
    if not w.is_cuda or w.dtype != torch.uint8 or w.numel() < nblocks * nbytes:
        raise ValueError('weights must be a CUDA uint8 tensor holding the blocks')
    out = torch.empty(tuple(shape), dtype=dtype, device=w.device)
    lib = _lib.load()
    if dtype == torch.float32:
        st = lib.b200q_dequant_f32_dev(ggml_type, w.data_ptr(), out.data_ptr(), nblocks, _stream())
    elif dtype == torch.bfloat16:
        st = lib.b200q_dequant_bf16_dev(ggml_type, w.data_ptr(), out.data_ptr(), nblocks, _stream())
    else:
        raise ValueError('dtype must be float32 or bfloat16')
    _lib.check(st)
    return out


def gemv(w: torch.Tensor, x: torch.Tensor, ggml_type: int, rows: int, cols: int,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ W^T with f32 accumulation.

    ``x`` is f32 [cols] or [tokens, cols]; the result is [rows] or
    [tokens, rows].  Suited to decode (1 token) and small batches.  Besides
    the block-quantised types, F32 (0) and F16 (1) rows are taken (cols a
    multiple of 8, 16-byte aligned).
    """
    _check_weights(w, ggml_type, rows, cols)
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.dtype != torch.float32 or x2.shape[-1] != cols or not x2.is_cuda or x2.device != w.device:
        raise ValueError('x must be a CUDA float32 tensor with cols columns, on the device of the weights')
    x2 = x2.contiguous()
    tokens = x2.shape[0]
    if out is None:
        out = torch.empty((tokens, rows), dtype=torch.float32, device=x2.device)
    elif (out.shape != (tokens, rows) or not out.is_contiguous() or out.dtype != torch.float32
          or out.device != x2.device):
        raise ValueError('out must be a contiguous f32 [tokens, rows] tensor on the device of x')
    st = _lib.load().b200q_gemv_dev(ggml_type, w.data_ptr(), x2.data_ptr(), out.data_ptr(),
                                    rows, cols, tokens, rows, 1, _stream())
    _lib.check(st)
    return out.reshape(rows) if squeeze else out


def tensor_core_min_tokens() -> int:
    """Token count from which batched quantised matmuls use the tensor cores
    (the library setting shared with the localai_*_matmul entry points)."""
    return int(_lib.load().b200q_matmul_tensor_core_min_tokens(-1))


def tensor_core_shape_ok(ggml_type: int, rows: int, cols: int) -> bool:
    """Q4_0/Q8_0/Q4_K/Q5_K/Q6_K weights the tensor-core GEMM can stream as packed rows."""
    if ggml_type not in (2, 8, 12, 13, 14) or rows % 128 or cols % 64 or cols % BLOCK[ggml_type][0]:
        return False
    return row_bytes(ggml_type, cols) % 16 == 0


def matmul(w: torch.Tensor, x: torch.Tensor, ggml_type: int, rows: int, cols: int) -> torch.Tensor:
    """f32 [tokens, rows] = x @ W^T for f32 x [tokens, cols]: the tensor-core
    GEMM (bf16 operands, f32 accumulation) for batches of at least
    ``tensor_core_min_tokens()`` tokens on supported weights, else the f32 GEMV."""
    _check_weights(w, ggml_type, rows, cols)
    x2 = x.reshape(-1, cols)
    T = x2.shape[0]
    nmin = tensor_core_min_tokens()
    if nmin <= 0 or T < nmin or not tensor_core_shape_ok(ggml_type, rows, cols) or w.data_ptr() % 16:
        return gemv(w, x2, ggml_type, rows, cols)
    if x2.dtype != torch.float32 or not x2.is_cuda:
        raise ValueError('x must be a CUDA float32 tensor with cols columns')
    off = torch.tensor([0, T], dtype=torch.int32, device=x2.device)
    return gemm_quant(x2.contiguous().to(torch.bfloat16), w, off, k=cols, n_feat=rows, w_rows_per_group=rows,
                      ggml_type=ggml_type, out_dtype=torch.float32)


def check_device_error() -> None:
    """Synchronise and raise if a kernel reported a timed-out wait or bad index."""
    code = _lib.load().b200q_check_device_error()
    if code:
        raise _lib.B200QError(f'kernel error word {code}')


def packed_row_bytes(ggml_type: int, k: int) -> int:
    """Bytes of one GGUF row of k values (rounded up to whole blocks)."""
    if ggml_type == 12:
        return (k + 255) // 256 * 144
    if ggml_type == 13:
        return (k + 255) // 256 * 176
    if ggml_type == 14:
        return (k + 255) // 256 * 210
    if ggml_type == 8:
        return (k + 31) // 32 * 34
    if ggml_type == 2:
        return (k + 31) // 32 * 18
    raise ValueError(f'unsupported ggml type {ggml_type} for the tensor-core path')


def pad_rows(w: torch.Tensor, rows: int, row_bytes: int) -> tuple[torch.Tensor, int]:
    """Copy of ``rows`` packed rows of ``row_bytes`` with each row padded to a
    multiple of 16 bytes (the tensor-core GEMM loads rows with TMA); returns
    (tensor, stride).  Rows already 16-byte sized are returned unchanged."""
    if row_bytes % 16 == 0:
        return w, row_bytes
    stride = (row_bytes + 15) // 16 * 16
    out = torch.zeros((rows, stride), dtype=torch.uint8, device=w.device)
    out[:, :row_bytes] = w.reshape(rows, row_bytes)
    return out.reshape(-1), stride


def gemm_quant(x_bf16: torch.Tensor, w: torch.Tensor, row_off: torch.Tensor, *, k: int, n_feat: int,
               w_rows_per_group: int, ggml_type: int = 12, w_row_bytes: int = 0, up_offset: int = -1,
               out: torch.Tensor | None = None, row_scale: torch.Tensor | None = None,
               act: torch.Tensor | None = None, group_w: torch.Tensor | None = None, n_weight_groups: int = 0,
               out_dtype=torch.float32, max_ctas: int = 0) -> torch.Tensor:
    """Grouped tensor-core GEMM with in-kernel dequantisation of Q4_K (12),
    Q5_K (13), Q6_K (14), Q8_0 (8) or Q4_0 (2) weights.

    ``x_bf16`` [rows, k] bf16 activations; group g owns rows
    ``row_off[g]:row_off[g+1]`` (int32 CUDA tensor, groups+1 entries) and the
    weight rows ``wg*w_rows_per_group ...`` of ``w`` (raw GGUF bytes,
    ``w_row_bytes`` apart, 0 = packed), with ``wg = group_w[g]`` when
    ``group_w`` is given (then ``w`` holds ``n_weight_groups`` weight groups),
    else ``wg = g``.  Plain mode (``up_offset < 0``) returns [rows, n_feat] in
    ``out_dtype`` (f32 or bf16); gate/up mode returns bf16 [rows, n_feat] =
    SiLU(gate) * up with up rows at ``f + up_offset``.
    """
    if x_bf16.dtype != torch.bfloat16 or not x_bf16.is_cuda or x_bf16.dim() != 2 or x_bf16.shape[1] != k:
        raise ValueError('x must be a CUDA bf16 [rows, k] tensor')
    if row_off.dtype != torch.int32 or not row_off.is_cuda:
        raise ValueError('row_off must be a CUDA int32 tensor')
    x_bf16 = x_bf16.contiguous()
    rows = x_bf16.shape[0]
    dev = x_bf16.device
    if row_off.device != dev:
        raise ValueError('row_off must be on the device of x')
    groups = row_off.numel() - 1
    wgroups = n_weight_groups if group_w is not None else groups
    if group_w is not None and (group_w.dtype != torch.int32 or group_w.numel() != groups or group_w.device != dev):
        raise ValueError('group_w must be an int32 tensor on the device of x with one entry per group')
    stride = w_row_bytes or packed_row_bytes(ggml_type, k)
    if (w.dtype != torch.uint8 or not w.is_cuda or w.device != dev
            or w.numel() < wgroups * w_rows_per_group * stride):
        raise ValueError('w must hold the weight groups as GGUF rows, on the device of x')
    if row_scale is not None and (row_scale.dtype != torch.float32 or row_scale.device != dev
                                  or not row_scale.is_contiguous() or row_scale.numel() < rows):
        raise ValueError('row_scale must be a contiguous f32 tensor with a value per row of x, on its device')

    def _rows_ok(t):
        # every output row and feature the kernel may store lies inside t (16-byte row stores)
        return t.device == dev and t.dim() == 2 and t.shape[0] >= rows and t.shape[1] >= n_feat and t.stride(1) == 1

    lib = _lib.load()
    gw = None if group_w is None else group_w.data_ptr()
    if up_offset >= 0:
        if act is None:
            act = torch.empty((rows, n_feat), dtype=torch.bfloat16, device=x_bf16.device)
        elif act.dtype != torch.bfloat16 or not _rows_ok(act):
            raise ValueError('act must be a bf16 [rows, n_feat] tensor (unit column stride) on the device of x')
        st = lib.b200q_gemm_dev(ggml_type, x_bf16.data_ptr(), rows, k, w.data_ptr(), w_row_bytes, groups,
                                w_rows_per_group, up_offset, n_feat, row_off.data_ptr(), gw, wgroups, None, 0, 0,
                                None, act.data_ptr(), act.stride(0), max_ctas, _stream())
        _lib.check(st)
        return act
    if out is None:
        out = torch.empty((rows, n_feat), dtype=out_dtype, device=x_bf16.device)
    if out.dtype not in (torch.float32, torch.bfloat16) or not _rows_ok(out):
        raise ValueError('out must be an f32 or bf16 [rows, n_feat] tensor (unit column stride) on the device of x')
    st = lib.b200q_gemm_dev(ggml_type, x_bf16.data_ptr(), rows, k, w.data_ptr(), w_row_bytes, groups,
                            w_rows_per_group, -1, n_feat, row_off.data_ptr(), gw, wgroups, out.data_ptr(),
                            1 if out.dtype == torch.bfloat16 else 0, out.stride(0),
                            None if row_scale is None else row_scale.data_ptr(), None, 0, max_ctas, _stream())
    _lib.check(st)
    return out


def gemm_q4k(x_bf16: torch.Tensor, w: torch.Tensor, row_off: torch.Tensor, **kw) -> torch.Tensor:
    """gemm_quant for Q4_K weights (packed rows)."""
    return gemm_quant(x_bf16, w, row_off, ggml_type=12, **kw)
