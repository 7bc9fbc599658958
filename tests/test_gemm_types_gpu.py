"""GPU tests of the tensor-core grouped GEMM on Q6_K, Q8_0, Q5_K and Q4_0 weights, and of
the Q6_K MoE block of the benchmark's configuration 3 (D=2048, E=16,
F=1024, top-2; T = 1, 64, 4096).

References as for Q4_K: the f32 product of the same bf16-rounded operands
(normwise <= 5e-4: a few weights may sit one bf16 ulp apart) and the float64
oracle ``dequantize(raw) @ x`` (normwise <= 1e-2, the bf16 tensor-core bar).
Q6_K rows of 1024 values (840 B) and Q4_0 rows of 640 values (360 B) are
not 16-byte sized and go through ``ops.pad_rows`` exactly as ``QuantMoE``
does.
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import ops, synth
from localai_b200.moe import QuantMoE

pytestmark = pytest.mark.gpu


def weights(rng, t, rows, k, full_scales=False):
    if t in (13, 2):                    # Q5_K / Q4_0: random block bytes, small fp16 scales
        return synth.make(rng, t, rows, k)
    if t == 14:
        raw = synth.q6_k(rng, rows, k)
        if full_scales:                 # int8 scales over the whole range, incl. -128 and 127
            b = np.frombuffer(bytearray(raw), np.uint8).reshape(rows, k // 256, 210).copy()
            sc = rng.integers(-128, 128, size=(rows, k // 256, 16)).astype(np.int8)
            sc[0, 0, 0], sc[0, 0, 1] = -128, 127
            b[:, :, 192:208] = sc.view(np.uint8)
            raw = b.reshape(-1).tobytes()
    else:
        raw = synth.q8_0(rng, rows, k)
    return raw


def ref_bf16(raw, t, rows, k, x_bf16):
    w = torch.from_numpy(o.dequantize(raw, t, (rows, k))).to(torch.bfloat16).float().cuda()
    return x_bf16.float() @ w.T


@pytest.mark.parametrize('t,k,full', [(14, 2048, False), (14, 1024, False), (14, 512, True), (8, 512, False),
                                      (8, 1024, False), (13, 2048, False), (13, 1024, False), (2, 512, False),
                                      (2, 768, False), (2, 640, False)])
def test_plain_grouped(t, k, full):
    rng = np.random.default_rng(t * 100 + k)
    n = 256
    sizes = [37, 0, 256, 300]
    g = len(sizes)
    raw = weights(rng, t, g * n, k, full)
    rb = ops.packed_row_bytes(t, k)
    w, stride = ops.pad_rows(torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda(), g * n, rb)
    rows = sum(sizes)
    x = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda()
    xb = x.to(torch.bfloat16)
    off = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device='cuda')
    out = ops.gemm_quant(xb, w, off, k=k, n_feat=n, w_rows_per_group=n, ggml_type=t, w_row_bytes=stride)
    torch.cuda.synchronize()
    ops.check_device_error()
    rawb = np.frombuffer(raw, np.uint8)
    for gi in range(g):
        a, b = int(off[gi]), int(off[gi + 1])
        if a == b:
            continue
        graw = rawb[gi * n * rb:(gi + 1) * n * rb].tobytes()
        ref = ref_bf16(graw, t, n, k, xb[a:b])
        err = ((out[a:b] - ref).abs().max() / ref.abs().max()).item()
        assert err < 5e-4, (gi, err)
        ref64 = o.matmul_f64(graw, t, n, k, x[a:b].cpu().numpy())
        assert o.normwise_rel_err(out[a:b].cpu().numpy(), ref64) < 1e-2


@pytest.mark.parametrize('t,k', [(14, 1024), (8, 768), (13, 1024), (2, 512)])
def test_gate_up(t, k):
    rng = np.random.default_rng(t + k)
    f = 128
    sizes = [70, 0, 300]
    g = len(sizes)
    raw = weights(rng, t, g * 2 * f, k)
    rb = ops.packed_row_bytes(t, k)
    w, stride = ops.pad_rows(torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda(), g * 2 * f, rb)
    rows = sum(sizes)
    xb = torch.from_numpy(rng.normal(size=(rows, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    off = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device='cuda')
    act = ops.gemm_quant(xb, w, off, k=k, n_feat=f, w_rows_per_group=2 * f, up_offset=f, ggml_type=t,
                         w_row_bytes=stride)
    torch.cuda.synchronize()
    ops.check_device_error()
    rawb = np.frombuffer(raw, np.uint8)
    for gi in range(g):
        a, b = int(off[gi]), int(off[gi + 1])
        if a == b:
            continue
        gu = ref_bf16(rawb[gi * 2 * f * rb:(gi + 1) * 2 * f * rb].tobytes(), t, 2 * f, k, xb[a:b])
        gate, up = gu[:, :f], gu[:, f:]
        ref = gate / (1 + torch.exp(-gate.clamp(-80, 80))) * up
        err = ((act[a:b].float() - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-2, (gi, err)


def config3_layer(rng, T):
    E, D, F, k = 16, 2048, 1024, 2
    gate_up = [synth.q6_k(rng, 2 * F, D) for _ in range(E)]
    down = [synth.q6_k(rng, D, F) for _ in range(E)]
    wr = rng.normal(0, 0.02, size=(E, D)).astype(np.float32)
    cat = lambda parts: torch.frombuffer(bytearray(b''.join(parts)), dtype=torch.uint8).cuda()
    layer = QuantMoE(torch.from_numpy(wr).cuda(), cat(gate_up), cat(down), d_model=D, d_ff=F, top_k=k,
                     ggml_type=14)
    return layer, wr, gate_up, down


@pytest.mark.parametrize('T', [1, 64, 4096])
def test_config3_q6k_moe(T):
    """Configuration 3 against the float64 oracle run with the GPU's routing
    (renormalised top-2).  At T = 4096 the oracle runs on a 256-token sample."""
    rng = np.random.default_rng(300 + T)
    layer, wr, gate_up, down = config3_layer(rng, T)
    h = rng.normal(size=(T, 2048)).astype(np.float32)
    hd = torch.from_numpy(h).cuda()
    y = layer(hd)
    torch.cuda.synchronize()
    ops.check_device_error()
    _, ids, w = layer.route(hd)
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    sample = np.arange(T) if T <= 256 else rng.choice(T, 256, replace=False)
    experts = [(gate_up[e], down[e]) for e in range(16)]
    ref = o.moe_forward_f64(h[sample], ids[sample], w[sample], experts, 14, 14, 2048, 1024, 1024)
    assert o.normwise_rel_err(y.cpu().numpy()[sample], ref) < 1e-2


@pytest.mark.parametrize('t', [13, 2])
def test_moe_layer_q5k_q4_0(t):
    """The MoE layer on Q5_K and Q4_0 experts (tensor-core path) against the
    float64 oracle with the GPU's routing."""
    rng = np.random.default_rng(500 + t)
    E, D, F, k, T = 8, 1024, 256, 2, 600
    gate_up = [synth.make(rng, t, 2 * F, D) for _ in range(E)]
    down = [synth.make(rng, t, D, F) for _ in range(E)]
    wr = rng.normal(0, D ** -0.5, size=(E, D)).astype(np.float32)
    cat = lambda parts: torch.frombuffer(bytearray(b''.join(parts)), dtype=torch.uint8).cuda()
    layer = QuantMoE(torch.from_numpy(wr).cuda(), cat(gate_up), cat(down), d_model=D, d_ff=F, top_k=k,
                     ggml_type=t)
    h = rng.normal(size=(T, D)).astype(np.float32)
    hd = torch.from_numpy(h).cuda()
    assert T * k > layer.small_slots
    y = layer(hd)
    torch.cuda.synchronize()
    ops.check_device_error()
    _, ids, w = layer.route(hd)
    ref = o.moe_forward_f64(h, ids.cpu().numpy(), w.cpu().numpy(), list(zip(gate_up, down)), t, t, D, F, F)
    assert o.normwise_rel_err(y.cpu().numpy(), ref) < 1e-2
