"""GPU tests of the tensor-core causal prefill attention (b200q_attn_prefill_tc_dev)
against a float64 restatement of engine/model.py:130-160 (forward_sequence:
softmax(q k^T / sqrt(hd)) v over cache positions 0 .. pos + t, grouped-query
heads), and against the f32 CUDA-core kernel (b200q_attn_prefill_dev).

Bar: normwise relative error <= 1e-2 (bf16 q, k, v and probabilities, f32
accumulation).  Cache rows past pos + T hold NaN: the kernel must not read
them.
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import _lib

pytestmark = pytest.mark.gpu
ERR_BAD_INDEX = 2


def attention_f64(q, kc, vc, p0, H, KV, hd):
    """q [T, H, hd], caches [S, KV, hd] -> [T, H * hd] (float64)."""
    T = q.shape[0]
    out = np.zeros((T, H, hd))
    grp = H // KV
    for h in range(H):
        g = h // grp
        k = kc[:p0 + T, g].astype(np.float64)
        v = vc[:p0 + T, g].astype(np.float64)
        s = q[:, h].astype(np.float64) @ k.T / np.sqrt(hd)
        mask = np.arange(p0 + T)[None, :] > (p0 + np.arange(T))[:, None]
        s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h] = p @ v
    return out.reshape(T, H * hd)


def run(T, p0, H, KV, hd=128, max_seq=None, seed=0):
    lib = _lib.load()
    rng = np.random.default_rng(seed)
    max_seq = max_seq or p0 + T + 37
    R = (H + 2 * KV) * hd
    qkv = rng.normal(size=(T, R)).astype(np.float32)
    kc = np.full((max_seq, KV, hd), np.nan, np.float32)
    vc = np.full((max_seq, KV, hd), np.nan, np.float32)
    kc[:p0 + T] = rng.normal(size=(p0 + T, KV, hd))
    vc[:p0 + T] = rng.normal(size=(p0 + T, KV, hd))
    dev = lambda a: torch.from_numpy(a).cuda()
    d_qkv, d_k, d_v = dev(qkv), dev(kc), dev(vc)
    pos = torch.tensor([p0], dtype=torch.int32, device='cuda')
    nbytes = lib.b200q_attn_prefill_tc_scratch_bytes(T, H, KV, hd, max_seq)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device='cuda')
    out = torch.zeros((T, H * hd), dtype=torch.bfloat16, device='cuda')
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.b200q_attn_prefill_tc_dev(d_qkv.data_ptr(), d_k.data_ptr(), d_v.data_ptr(), pos.data_ptr(), T, H,
                                             KV, hd, max_seq, scratch.data_ptr(), nbytes, out.data_ptr(), st))
    torch.cuda.synchronize()
    code = lib.b200q_check_device_error()
    return out, code, qkv, kc, vc, (d_qkv, d_k, d_v, pos)


@pytest.mark.parametrize('T,p0,H,KV', [(128, 0, 8, 2), (200, 0, 8, 2), (300, 77, 8, 2), (1024, 0, 8, 2),
                                       (512, 0, 32, 8), (5, 250, 4, 4), (129, 1, 4, 1),
                                       (2048, 0, 32, 8)])          # configuration 4's prompt and heads
def test_tc_prefill_matches_f64(T, p0, H, KV):
    hd = 128
    out, code, qkv, kc, vc, _ = run(T, p0, H, KV, hd, seed=T + p0)
    assert code == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    ref = attention_f64(qkv[:, :H * hd].reshape(T, H, hd), kc, vc, p0, H, KV, hd)
    assert o.normwise_rel_err(got, ref) < 1e-2


def test_tc_prefill_matches_cuda_core_kernel():
    T, p0, H, KV, hd = 384, 40, 16, 4, 128
    out, code, _, _, _, (d_qkv, d_k, d_v, pos) = run(T, p0, H, KV, hd, seed=9)
    assert code == 0
    lib = _lib.load()
    max_seq = d_k.shape[0]
    ref = torch.zeros_like(out)
    _lib.check(lib.b200q_attn_prefill_dev(d_qkv.data_ptr(), d_k.data_ptr(), d_v.data_ptr(), pos.data_ptr(), T, H, KV,
                                          hd, max_seq, ref.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert o.normwise_rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy()) < 1e-2


def test_tc_prefill_out_of_range_position_reports():
    """pos + T beyond the cache: nothing written, the error word says so."""
    lib = _lib.load()
    T, H, KV, hd, max_seq = 64, 4, 2, 128, 100
    d_qkv = torch.zeros((T, (H + 2 * KV) * hd), device='cuda')
    d_k = torch.zeros((max_seq, KV, hd), device='cuda')
    d_v = torch.zeros_like(d_k)
    pos = torch.tensor([50], dtype=torch.int32, device='cuda')
    nbytes = lib.b200q_attn_prefill_tc_scratch_bytes(T, H, KV, hd, max_seq)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device='cuda')
    out = torch.full((T, H * hd), 7.0, dtype=torch.bfloat16, device='cuda')
    _lib.check(lib.b200q_attn_prefill_tc_dev(d_qkv.data_ptr(), d_k.data_ptr(), d_v.data_ptr(), pos.data_ptr(), T, H,
                                             KV, hd, max_seq, scratch.data_ptr(), nbytes, out.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert lib.b200q_check_device_error() == ERR_BAD_INDEX
    assert bool((out == 7.0).all())
