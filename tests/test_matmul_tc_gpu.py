"""The reference's batched matmul boundary on the tensor cores.

``localai_{q4k,q5k,q6k,q8_0,q4_0}_matmul`` (engine/native_quant.cpp:749-768, the
prefill path decoded_matmul_row :620-703) called through ctypes with host
buffers -- exactly as engine/native_quant.py:130-156 does -- and
``DeviceGGUF.matmul`` (engine/gguf_parser.py:290-331) run the tcgen05 GEMM for
batches of at least ``b200q_matmul_tensor_core_min_tokens`` tokens: bf16
operands, f32 accumulation, bar 1e-2 normwise against ``matmul_f64``.  Output
in the reference's [rows][tokens] layout (transposed by the Python wrapper
to [tokens, rows], as the reference does).  Shapes the GEMM cannot take and
batches below the threshold stay on the f32 GEMV (bar 1e-3).
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import _lib, native_quant, synth

pytestmark = pytest.mark.gpu


def _launches():
    return _lib.launch_count()


@pytest.mark.parametrize('t,rows,cols,tokens', [(12, 14336, 4096, 512), (12, 4096, 14336, 512),
                                                (14, 1024, 2048, 333), (8, 1024, 4096, 77),
                                                (12, 256, 1536, 32), (8, 128, 256, 300),
                                                (13, 512, 2048, 100), (2, 256, 1024, 64)])
def test_drop_in_matmul_on_tensor_cores(t, rows, cols, tokens):
    lib = _lib.load()
    assert lib.b200q_matmul_tensor_core_min_tokens(-1) == 32
    rng = np.random.default_rng(rows + cols + tokens + t)
    raw = synth.make(rng, t, rows, cols) if t != 12 else synth.q4_k(rng, rows, cols)
    x = rng.normal(size=(tokens, cols)).astype(np.float32)
    n0 = _launches()
    got = native_quant.matmul(raw, x, rows, cols, t, 8)
    assert _launches() - n0 == 2                   # bf16 conversion + tcgen05 GEMM
    assert got.shape == (tokens, rows) and got.dtype == np.float32
    err = o.normwise_rel_err(got, o.matmul_f64(raw, t, rows, cols, x))
    assert err <= 1e-2, err


def test_threshold_and_ineligible_shapes_use_the_gemv():
    lib = _lib.load()
    rng = np.random.default_rng(9)
    cases = [(12, 200, 1024, 64),        # rows not a multiple of 128
             (14, 128, 1024, 64),        # Q6_K rows of 840 bytes (not whole 16-byte units)
             (2, 128, 1056, 64),         # Q4_0 rows of 594 bytes (not whole 16-byte units)
             (12, 256, 1024, 31)]        # below the threshold
    for t, rows, cols, tokens in cases:
        raw = synth.make(rng, t, rows, cols)
        x = rng.normal(size=(tokens, cols)).astype(np.float32)
        n0 = _launches()
        got = native_quant.matmul(raw, x, rows, cols, t)
        assert _launches() - n0 == 1
        assert o.normwise_rel_err(got, o.matmul_f64(raw, t, rows, cols, x)) <= 1e-3
    prev = lib.b200q_matmul_tensor_core_min_tokens(0)      # everything on the f32 GEMV
    try:
        raw = synth.q4_k(rng, 256, 1024)
        x = rng.normal(size=(100, 1024)).astype(np.float32)
        got = native_quant.matmul(raw, x, 256, 1024, 12)
        assert o.normwise_rel_err(got, o.matmul_f64(raw, 12, 256, 1024, x)) <= 1e-3
    finally:
        assert lib.b200q_matmul_tensor_core_min_tokens(prev) == 0


def test_registered_weights_and_device_gguf_matmul(tmp_path):
    """A registered host range (the GGUF mmap) and DeviceGGUF.matmul take the
    same tensor-core path."""
    from localai_b200.gguf import DeviceGGUF, write_gguf
    rng = np.random.default_rng(12)
    rows, cols, T = 512, 2048, 96
    raw = synth.q4_k(rng, rows, cols)
    path = tmp_path / 'm.gguf'
    write_gguf(path, {'general.architecture': 'llama'}, {'blk.0.ffn_up.weight': (raw, 12, (rows, cols))})
    g = DeviceGGUF(path)
    X = rng.normal(size=(T, cols)).astype(np.float32)
    ref = o.matmul_f64(raw, 12, rows, cols, X)
    Y = g.matmul('blk.0.ffn_up.weight', torch.from_numpy(X).cuda())
    assert Y.shape == (T, rows)
    assert o.normwise_rel_err(Y.cpu().numpy(), ref) <= 1e-2
    buf = bytearray(raw)
    addr = native_quant.register_weights(buf)
    try:
        got = native_quant.matmul(buf, X, rows, cols, 12)
        assert o.normwise_rel_err(got, ref) <= 1e-2
    finally:
        native_quant.unregister_weights(addr)
