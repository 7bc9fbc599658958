"""GPU tests of the tcgen05 grouped GEMM with in-kernel Q4_K dequantisation.

Two references: (1) the same bf16-rounded operands multiplied in f32 by
torch (isolates the tensor-core path: tight tolerance), (2) the f64 oracle
``dequantize(raw) @ x`` with f32 activations (the bf16 tensor-core path bar:
normwise max relative error <= 1e-2).
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import ops, synth

pytestmark = pytest.mark.gpu


def q4k_weights(rng, rows, k, zero_tail=0):
    kpad = (k + 255) // 256 * 256
    raw = synth.q4_k(rng, rows, kpad, zero_tail_cols=zero_tail)
    return raw, torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda(), kpad


def ref_bf16(raw, rows, kpad, k, x_bf16):
    """f32 product of the bf16-rounded exact weights and the bf16 activations."""
    w = torch.from_numpy(o.dequantize(raw, 12, (rows, kpad))[:, :k]).to(torch.bfloat16).float().cuda()
    return x_bf16.float() @ w.T


@pytest.mark.parametrize('sizes', [[300], [0, 1, 255, 256, 257, 600, 0, 31]])
def test_plain_grouped_matches_reference(sizes):
    rng = np.random.default_rng(len(sizes))
    k, n = 512, 256
    g = len(sizes)
    raw, w, kpad = q4k_weights(rng, g * n, k)
    rows = sum(sizes)
    x = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda()
    xb = x.to(torch.bfloat16)
    off = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device='cuda')
    scale = torch.from_numpy(rng.uniform(0.5, 1.5, size=rows).astype(np.float32)).cuda()
    out = ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, row_scale=scale)
    torch.cuda.synchronize()
    ops.check_device_error()
    rawb = np.frombuffer(raw, np.uint8)
    rb = (kpad // 256) * 144
    for gi in range(g):
        a, b = int(off[gi]), int(off[gi + 1])
        if a == b:
            continue
        graw = rawb[gi * n * rb:(gi + 1) * n * rb].tobytes()
        ref = ref_bf16(graw, n, kpad, k, xb[a:b]) * scale[a:b, None]
        got = out[a:b]
        err = ((got - ref).abs().max() / ref.abs().max()).item()
        assert err < 5e-4, (gi, err)   # a few weights can sit one bf16 ulp apart
        ref64 = o.matmul_f64(graw, 12, n, kpad, x[a:b].cpu().numpy()) * scale[a:b, None].cpu().numpy()
        assert o.normwise_rel_err(got.cpu().numpy(), ref64) < 1e-2


def test_gate_up_fused_silu():
    rng = np.random.default_rng(7)
    k, f = 768, 128
    sizes = [70, 300, 0, 513]
    g = len(sizes)
    raw, w, kpad = q4k_weights(rng, g * 2 * f, k)
    rows = sum(sizes)
    x = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda()
    xb = x.to(torch.bfloat16)
    off = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device='cuda')
    act = ops.gemm_q4k(xb, w, off, k=k, n_feat=f, w_rows_per_group=2 * f, up_offset=f)
    torch.cuda.synchronize()
    ops.check_device_error()
    rawb = np.frombuffer(raw, np.uint8)
    rb = (kpad // 256) * 144
    for gi in range(g):
        a, b = int(off[gi]), int(off[gi + 1])
        if a == b:
            continue
        graw = rawb[gi * 2 * f * rb:(gi + 1) * 2 * f * rb].tobytes()
        gu = ref_bf16(graw, 2 * f, kpad, k, xb[a:b])
        gate, up = gu[:, :f], gu[:, f:]
        ref = gate / (1 + torch.exp(-gate.clamp(-80, 80))) * up
        err = ((act[a:b].float() - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-2, (gi, err)


def test_k_not_multiple_of_256():
    """K = 1408 (config 5 down projection): weights padded to 1536 with zero sub-blocks."""
    rng = np.random.default_rng(9)
    k, n, rows = 1408, 128, 200
    raw, w, kpad = q4k_weights(rng, n, k, zero_tail=128)
    x = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda()
    xb = x.to(torch.bfloat16)
    off = torch.tensor([0, rows], dtype=torch.int32, device='cuda')
    out = ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n)
    torch.cuda.synchronize()
    ref = ref_bf16(raw, n, kpad, k, xb)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 5e-4
    xp = np.zeros((rows, kpad), np.float32)
    xp[:, :k] = x.cpu().numpy()
    assert o.normwise_rel_err(out.cpu().numpy(), o.matmul_f64(raw, 12, n, kpad, xp)) < 1e-2


def test_large_k_many_tiles():
    rng = np.random.default_rng(11)
    k, n, rows = 4096, 512, 1500
    raw, w, kpad = q4k_weights(rng, n, k)
    xb = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    off = torch.tensor([0, rows], dtype=torch.int32, device='cuda')
    out = ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, max_ctas=7)
    torch.cuda.synchronize()
    ops.check_device_error()
    ref = ref_bf16(raw, n, kpad, k, xb)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 5e-4


def test_group_weight_map_and_bf16_output():
    """Groups that reuse weight groups out of order (the expert-parallel
    layout: one group per (source rank, local expert)), bf16 rows out."""
    rng = np.random.default_rng(13)
    k, n = 512, 128
    n_w = 3
    raw, w, kpad = q4k_weights(rng, n_w * n, k)
    sizes = [100, 0, 300, 17, 256]
    gmap = [2, 0, 2, 1, 0]
    rows = sum(sizes)
    xb = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    off = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device='cuda')
    gw = torch.tensor(gmap, dtype=torch.int32, device='cuda')
    scale = torch.from_numpy(rng.uniform(0.5, 1.5, size=rows).astype(np.float32)).cuda()
    out = ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, row_scale=scale, group_w=gw,
                       n_weight_groups=n_w, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    ops.check_device_error()
    rawb = np.frombuffer(raw, np.uint8)
    rb = (kpad // 256) * 144
    for g, wg in enumerate(gmap):
        a, b = int(off[g]), int(off[g + 1])
        if a == b:
            continue
        graw = rawb[wg * n * rb:(wg + 1) * n * rb].tobytes()
        ref = ref_bf16(graw, n, kpad, k, xb[a:b]) * scale[a:b, None]
        err = ((out[a:b].float() - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-2, (g, err)


def test_wrappers_refuse_host_or_short_buffers():
    """ops.gemm_quant / ops.gemv refuse an output, activation or scale buffer
    in host memory or too small for the rows and features the kernel stores
    (ValueError before any launch, instead of a device fault)."""
    rng = np.random.default_rng(3)
    k, n, rows = 512, 128, 40
    raw, w, kpad = q4k_weights(rng, 2 * n, k)
    xb = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    off = torch.tensor([0, rows], dtype=torch.int32, device='cuda')
    for bad in (torch.empty((rows, n)), torch.empty((rows - 1, n), device='cuda'),
                torch.empty((rows, n - 8), device='cuda'), torch.empty((n, rows), device='cuda').t()):
        with pytest.raises(ValueError):
            ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, out=bad)
    with pytest.raises(ValueError):
        ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=2 * n, up_offset=n,
                     act=torch.empty((rows, n), dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, row_scale=torch.ones(rows - 1, device='cuda'))
    x = torch.zeros((1, k), device='cuda')
    with pytest.raises(ValueError):
        ops.gemv(w, x, 12, n, k, out=torch.empty((1, n)))
    ok = ops.gemm_q4k(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, out=torch.empty((rows, n), device='cuda'))
    torch.cuda.synchronize()
    assert ok.shape == (rows, n)
