"""GPU parity tests of the dequant and GEMV kernels against the CPU oracle.

Bars: dequant bit-exact; GEMV/matmul normwise max relative error <= 1e-3
against ``dequantize(raw) @ x`` in float64 (f32-accumulate path).  The
reference-style cases (rows=300 > 256, cols=512, seeds 50-55) mirror
tests/test_dequant.py:119-230 of the reference, whose elementwise tolerances
(rtol 2e-4/3e-4, atol 2e-3/3e-3) are checked as well.
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import native_quant, ops, synth

pytestmark = pytest.mark.gpu
TOL = 1e-3
TYPES = (2, 8, 12, 13, 14)


def dev_bytes(raw, offset=0):
    buf = torch.zeros(len(raw) + offset + 64, dtype=torch.uint8)
    buf[offset:offset + len(raw)] = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
    return buf.cuda()[offset:offset + len(raw)]


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_dequant_golden_bit_exact(golden):
    for name, t, rows, cols, raw, ref in golden:
        if t not in TYPES:
            continue
        got = ops.dequantize(dev_bytes(raw), t, (rows, cols)).cpu().numpy()
        assert np.array_equal(bits(got), bits(ref)), name


@pytest.mark.parametrize('t', TYPES)
def test_dequant_large_bit_exact(t):
    rng = np.random.default_rng(100 + t)
    rows, cols = 512, 4096
    raw = synth.make(rng, t, rows, cols)
    got = ops.dequantize(dev_bytes(raw), t, (rows, cols)).cpu().numpy()
    assert np.array_equal(bits(got), bits(o.dequantize(raw, t, (rows, cols))))
    gb = ops.dequantize(dev_bytes(raw), t, (rows, cols), dtype=torch.bfloat16).float().cpu().numpy()
    ref_bf16 = torch.from_numpy(o.dequantize(raw, t, (rows, cols))).to(torch.bfloat16).float().numpy()
    assert np.array_equal(gb, ref_bf16)


@pytest.mark.parametrize('t,seed', [(8, 50), (2, 55), (13, 54), (12, 51), (14, 52)])
def test_reference_style_matvec(t, seed):
    rng = np.random.default_rng(seed)
    rows, cols = 300, 512
    raw = synth.random_blocks(rng, t, rows, cols, d=0.0005 if t in (12, 13, 14) else 0.03125, dmin=0.00025)
    x = rng.normal(size=cols).astype(np.float32)
    ref = o.matvec_f64(raw, t, rows, cols, x)
    for threads in (1, 4, 8):
        got = native_quant.matvec(raw, x, rows, cols, t, threads)
        assert got.dtype == np.float32 and got.shape == (rows,)
        np.testing.assert_allclose(got, ref, rtol=2e-4, atol=2e-3)
        assert o.normwise_rel_err(got, ref) <= TOL


def test_reference_style_batched_matmul():
    """tests/test_dequant.py:160-177: all five types, 5 tokens."""
    rng = np.random.default_rng(53)
    rows, cols, tokens = 300, 512, 5
    vectors = rng.normal(size=(tokens, cols)).astype(np.float32)
    for t in TYPES:
        raw = synth.random_blocks(rng, t, rows, cols)
        ref = o.matmul_f64(raw, t, rows, cols, vectors)
        got = native_quant.matmul(raw, vectors, rows, cols, t, 4)
        assert got.shape == (tokens, rows)
        np.testing.assert_allclose(got, ref, rtol=3e-4, atol=3e-3, err_msg=f'type {t}')
        assert o.normwise_rel_err(got, ref) <= TOL


def test_q4_0_varied_sizes_and_nibble_edges():
    """tests/test_dequant.py:179-200: cols 32..512, zero/tiny/unit scales, nibble extremes."""
    rng = np.random.default_rng(551)
    for cols in (32, 64, 96, 512):
        rows, nb = 300, cols // 32
        blocks = rng.integers(0, 256, size=(rows, nb, 18), dtype=np.uint8)
        for r in range(rows):
            for b in range(nb):
                blocks[r, b, 0:2] = np.frombuffer(np.float16((0.0, 0.0001, 0.03125, 1.0)[(r + b) % 4]).tobytes(), np.uint8)
                if r % 3 == 0:
                    blocks[r, b, 2:18] = np.frombuffer(bytes([0x07, 0x80, 0xF8, 0xFF]) * 4, np.uint8)
        raw = blocks.tobytes()
        x = rng.normal(size=cols).astype(np.float32)
        ref = o.matvec_f64(raw, 2, rows, cols, x)
        got = native_quant.matvec(raw, x, rows, cols, 2, 4)
        np.testing.assert_allclose(got, ref, rtol=2e-4, atol=2e-3, err_msg=f'cols={cols}')


@pytest.mark.parametrize('t', TYPES)
@pytest.mark.parametrize('rows,cols', [(1, 256), (7, 512), (33, 768), (100, 1024), (257, 2048), (64, 14336)])
def test_matvec_shapes(t, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols + t)
    raw = synth.make(rng, t, rows, cols)
    x = rng.normal(size=cols).astype(np.float32)
    got = native_quant.matvec(raw, x, rows, cols, t)
    assert o.normwise_rel_err(got, o.matvec_f64(raw, t, rows, cols, x)) <= TOL


@pytest.mark.parametrize('t', TYPES)
@pytest.mark.parametrize('tokens', [2, 3, 4, 5, 8, 13])
def test_small_batch_matmul(t, tokens):
    rng = np.random.default_rng(tokens * 31 + t)
    rows, cols = 160, 1024
    raw = synth.make(rng, t, rows, cols)
    x = rng.normal(size=(tokens, cols)).astype(np.float32)
    got = native_quant.matmul(raw, x, rows, cols, t)
    assert o.normwise_rel_err(got, o.matmul_f64(raw, t, rows, cols, x)) <= TOL


@pytest.mark.parametrize('t', (12, 14, 8))
def test_config1_size_4096(t):
    """Config 1 shape (4096 x 4096), benchmark value distributions."""
    rng = np.random.default_rng(1)
    raw = synth.make(rng, t, 4096, 4096)
    x = rng.normal(size=4096).astype(np.float32)
    got = native_quant.matvec(raw, x, 4096, 4096, t)
    assert o.normwise_rel_err(got, o.matvec_f64(raw, t, 4096, 4096, x)) <= TOL


@pytest.mark.parametrize('rows', (4096, 14336))
def test_q4k_batch1_tensor_core_and_cuda_core_paths(rows):
    """Batch-1 Q4_K at the benchmark's GEMV shapes through both kernels: the
    integer-tensor-core kernel (the default; x on a 16-bit grid per 256
    values, so its error is a few 1e-5) and the CUDA-core dp4a kernel (x on a
    22-bit grid, error near f32 rounding).  The profiler's kernel list shows
    which one ran."""
    from torch.profiler import ProfilerActivity, profile
    rng = np.random.default_rng(rows)
    cols = 4096
    raw = synth.q4_k(rng, rows, cols)
    w = dev_bytes(raw)
    xh = rng.normal(size=cols).astype(np.float32)
    x = torch.from_numpy(xh).cuda().view(1, cols)
    ref = o.matvec_f64(raw, 12, rows, cols, xh)
    lib = ops._lib.load()
    bounds = {1: 2e-4, 0: 2e-5}
    try:
        for enable, bound in bounds.items():
            lib.b200q_gemv_mma_tuning(enable, 0, 0, -1)
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                y = ops.gemv(w, x, 12, rows, cols)
                torch.cuda.synchronize()
            ops.check_device_error()
            names = [e.key for e in prof.key_averages() if 'gemv' in e.key]
            assert names and all(('gemv_q4k_mma_kernel' in n) == bool(enable) for n in names), names
            assert o.normwise_rel_err(y.cpu().numpy()[0], ref) <= bound
    finally:
        lib.b200q_gemv_mma_tuning(1, 0, 0, -1)


@pytest.mark.parametrize('t', (12, 14))
@pytest.mark.parametrize('offset', (2, 6, 10))
def test_device_api_unaligned_weight_base(t, offset):
    """Weights that start at a 2-byte (not 16-byte) aligned device address,
    e.g. an expert slice of a larger tensor."""
    rng = np.random.default_rng(offset + t)
    rows, cols = 96, 1024
    raw = synth.make(rng, t, rows, cols)
    w = dev_bytes(raw, offset)
    assert w.data_ptr() % 16 == offset % 16
    x = torch.from_numpy(rng.normal(size=(3, cols)).astype(np.float32)).cuda()
    y = ops.gemv(w, x, t, rows, cols)
    torch.cuda.synchronize()
    ops.check_device_error()
    assert o.normwise_rel_err(y.cpu().numpy(), o.matmul_f64(raw, t, rows, cols, x.cpu().numpy())) <= TOL


def test_registered_weights_path():
    rng = np.random.default_rng(9)
    rows, cols = 512, 2048
    raw = bytearray(synth.make(rng, 12, rows, cols))
    addr = native_quant.register_weights(raw)
    try:
        x = rng.normal(size=cols).astype(np.float32)
        got = native_quant.matvec(raw, x, rows, cols, 12)
        assert o.normwise_rel_err(got, o.matvec_f64(bytes(raw), 12, rows, cols, x)) <= TOL
    finally:
        native_quant.unregister_weights(addr)


def test_deterministic_repeat():
    rng = np.random.default_rng(11)
    raw = synth.make(rng, 12, 1024, 4096)
    x = rng.normal(size=4096).astype(np.float32)
    a = native_quant.matvec(raw, x, 1024, 4096, 12)
    b = native_quant.matvec(raw, x, 1024, 4096, 12)
    assert np.array_equal(bits(a), bits(b))

