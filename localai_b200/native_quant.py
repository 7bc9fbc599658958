"""Drop-in replacement for the reference's ``engine/native_quant.py``.

Same functions, signatures and conventions as the reference module
(engine/native_quant.py:66-156), backed by the B200 library instead of the
AVX2 DLL:

* ``get_native()`` returns the loaded library (ctypes CDLL) with the ten
  ``localai_*`` argtypes set, exactly as the reference binds them (:76-94).
  Unlike the reference, a missing library is an error, not ``None``: this
  package has no CPU fallback, and it says so loudly.
* ``matvec(raw, x, rows, cols, ggml_type, threads=4)`` -> f32[rows] (:102-126)
* ``matmul(raw, vectors, rows, cols, ggml_type, threads=4)`` -> f32[T, rows]
  (:130-156; the library writes [rows, T] like the reference kernel and the
  transpose happens here, as there).

``None`` is still returned where the reference returns it for a shape or type
the kernels do not handle (types outside {2, 8, 12, 13, 14}, ``rows < 1``,
``cols`` not a positive multiple of the block), and ``ValueError`` is raised
for byte-size mismatches with the reference's messages.  A kernel or CUDA
failure raises ``B200QError``.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

_BYTES = {2: 18, 8: 34, 12: 144, 13: 176, 14: 210}
_MATVEC = {2: 'localai_q4_0_matvec', 8: 'localai_q8_0_matvec', 12: 'localai_q4k_matvec',
           13: 'localai_q5k_matvec', 14: 'localai_q6k_matvec'}
_MATMUL = {2: 'localai_q4_0_matmul', 8: 'localai_q8_0_matmul', 12: 'localai_q4k_matmul',
           13: 'localai_q5k_matmul', 14: 'localai_q6k_matmul'}


def get_native():
    """The loaded libb200quant (engine/native_quant.py:66-99 contract, minus the None)."""
    return _lib.load()


def _block(ggml_type):
    return 32 if ggml_type in (2, 8) else 256


def matvec(raw, x: np.ndarray, rows: int, cols: int, ggml_type: int, threads: int = 4):
    """Quantized matvec W[rows, cols] @ x (engine/native_quant.py:102-126)."""
    if ggml_type not in _MATVEC or rows < 1:
        return None
    block_size = _block(ggml_type)
    if cols < block_size or cols % block_size:
        return None
    lib = get_native()
    raw_view = np.frombuffer(raw, dtype=np.uint8)
    expected_bytes = rows * (cols // block_size) * _BYTES[ggml_type]
    if raw_view.size != expected_bytes or np.asarray(x).size != cols:
        raise ValueError('native quantized matvec received an invalid tensor or vector size')
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(rows, dtype=np.float32)
    getattr(lib, _MATVEC[ggml_type])(
        raw_view.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
        x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
        int(rows), int(cols), int(threads))
    _lib.check()
    return out


def matmul(raw, vectors: np.ndarray, rows: int, cols: int, ggml_type: int, threads: int = 4):
    """Batched quantized matmul -> [tokens, rows] (engine/native_quant.py:130-156)."""
    if ggml_type not in _MATMUL or rows < 1:
        return None
    block_size = _block(ggml_type)
    if cols < block_size or cols % block_size:
        return None
    lib = get_native()
    x = np.ascontiguousarray(vectors, dtype=np.float32)
    if x.ndim != 2 or x.shape[1] != cols or x.shape[0] < 1:
        raise ValueError('native quantized matmul received an invalid input matrix')
    raw_view = np.frombuffer(raw, dtype=np.uint8)
    expected_bytes = rows * (cols // block_size) * _BYTES[ggml_type]
    if raw_view.size != expected_bytes:
        raise ValueError('native quantized matmul received an invalid tensor size')
    out = np.empty((rows, x.shape[0]), dtype=np.float32)
    getattr(lib, _MATMUL[ggml_type])(
        raw_view.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
        x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
        int(rows), int(cols), int(x.shape[0]), int(threads))
    _lib.check()
    return out.T.copy()


def register_weights(buffer) -> int:
    """Upload an immutable host buffer once (e.g. a GGUF mmap); later
    matvec/matmul calls on bytes inside it skip the weight copy.  Returns the
    host address used as the registry key."""
    view = np.frombuffer(buffer, dtype=np.uint8)
    addr = view.ctypes.data
    _lib.check(get_native().b200q_register_host(ctypes.c_void_p(addr), view.size))
    return addr


def unregister_weights(addr: int) -> None:
    _lib.check(get_native().b200q_unregister_host(ctypes.c_void_p(addr)))
