"""GPU tests of the MoE layer: routing, dispatch, expert products, combine.

* top-k: bit-exact expert ids against the oracle on the same logits
  (engine/zaya.py:290-296 generalised to top-k), weights to 1e-6;
* router logits against float64;
* dispatch: stable counting sort (slot order follows token order inside an
  expert), gathered rows equal bf16(h[token]);
* the whole layer against ``moe_forward_f64`` run with the GPU's routing
  decisions: normwise max relative error <= 1e-2 (bf16 tensor-core path).
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import synth
from localai_b200.moe import QuantMoE, chunk_bounds

pytestmark = pytest.mark.gpu

# Routing decisions may differ from float64 ones only where the oracle's k-th
# and (k+1)-th probabilities are closer than this (the router's f32 dot
# products move a logit by ~1e-6, a probability by less; 2e-6 leaves a
# twentyfold allowance and is far below the typical margin).
ROUTE_MARGIN = 2e-6


def make_layer(rng, E, D, F, k, renorm=True, router_bias=None, sel_bias=None):
    F_pad = (F + 255) // 256 * 256
    gate_up = [synth.q4_k(rng, 2 * F, D) for _ in range(E)]
    down = [synth.q4_k(rng, D, F_pad, zero_tail_cols=F_pad - F) for _ in range(E)]
    wr = rng.normal(0, 1 / np.sqrt(D), size=(E, D)).astype(np.float32)
    cat = lambda parts: torch.frombuffer(bytearray(b''.join(parts)), dtype=torch.uint8).cuda()
    layer = QuantMoE(torch.from_numpy(wr).cuda(), cat(gate_up), cat(down), d_model=D, d_ff=F, top_k=k,
                     router_bias=None if router_bias is None else torch.from_numpy(router_bias).cuda(),
                     sel_bias=None if sel_bias is None else torch.from_numpy(sel_bias).cuda(), renormalize=renorm)
    return layer, wr, gate_up, down, F_pad


@pytest.mark.parametrize('E,k,renorm,bias', [(64, 8, True, False), (16, 2, True, False), (17, 1, False, True),
                                             (128, 4, True, True), (8, 8, True, False)])
def test_topk_bit_exact_on_oracle_logits(E, k, renorm, bias):
    rng = np.random.default_rng(E * 10 + k)
    T = 700
    logits = rng.normal(size=(T, E)).astype(np.float32)
    logits[5, :] = 0.0                        # all-tie row: lower indices win
    logits[6, 1] = logits[6, E - 1] = 5.0     # a two-way tie at the top
    sel_bias = rng.normal(scale=0.05, size=E).astype(np.float32) if bias else None
    ref_ids, ref_w = o.route_topk(logits, k, bias=sel_bias, renormalize=renorm)
    layer = QuantMoE.__new__(QuantMoE)
    layer.E, layer.k, layer.renorm = E, k, 1 if renorm else 0
    layer.sel_bias = None if sel_bias is None else torch.from_numpy(sel_bias).cuda()
    from localai_b200 import _lib
    layer.lib = _lib.load()
    ids, w = layer.topk(torch.from_numpy(logits).cuda())
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(w.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize('T,E,D', [(1, 64, 4096), (7, 64, 4096), (37, 100, 2048), (300, 64, 4096),
                                   (4096, 64, 2048), (65, 17, 516)])
def test_fused_route_split_and_unsplit(T, E, D):
    """b200q_moe_route_dev: split-K (few tokens) and single-pass (many tokens)
    logits against float64; its ids/weights equal the top-k kernel run on the
    logits it returns; two calls agree bit for bit."""
    from localai_b200 import _lib
    rng = np.random.default_rng(T * 7 + E)
    k = 4
    wr = rng.normal(0, 1 / np.sqrt(D), size=(E, D)).astype(np.float32)
    bias = rng.normal(scale=0.1, size=E).astype(np.float32)
    h = rng.normal(size=(T, D)).astype(np.float32)
    layer = QuantMoE.__new__(QuantMoE)
    layer.lib = _lib.load()
    layer.E, layer.D, layer.k, layer.renorm = E, D, k, 1
    layer.router_w = torch.from_numpy(wr).cuda()
    layer.router_bias = torch.from_numpy(bias).cuda()
    layer.sel_bias = None
    hd = torch.from_numpy(h).cuda()
    logits, ids, w = layer.route(hd)
    ref = h.astype(np.float64) @ wr.T.astype(np.float64) + bias
    err = np.abs(logits.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
    ids2, w2 = layer.topk(logits)
    assert torch.equal(ids, ids2) and torch.equal(w, w2)
    logits3, ids3, w3 = layer.route(hd)
    assert torch.equal(logits, logits3) and torch.equal(ids, ids3) and torch.equal(w, w3)
    # the separate router entry: same bar; identical when the fused call did not split
    plain = torch.empty_like(logits)
    _lib.check(layer.lib.b200q_moe_router_dev(hd.data_ptr(), layer.router_w.data_ptr(), layer.router_bias.data_ptr(),
                                              plain.data_ptr(), T, E, D, torch.cuda.current_stream().cuda_stream))
    err = np.abs(plain.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
    if layer.lib.b200q_moe_route_workspace_bytes(T, E, D) == 0:
        assert torch.equal(plain, logits)


@pytest.mark.parametrize('T,E,D', [(2048, 64, 4096), (16384, 64, 4096), (1000, 40, 1056), (129, 64, 4096),
                                   (64, 64, 4096)])
def test_router_accuracy_and_bf16_copy(T, E, D):
    """Router logits within 1e-6 of the float64 product relative to the
    largest logit, at the headline shape (16384 tokens, one pass) and split
    K (few tokens), and the bf16 copy of h written on the way equals bf16(h)."""
    from localai_b200 import _lib
    rng = np.random.default_rng(T + E)
    layer = QuantMoE.__new__(QuantMoE)
    layer.lib = _lib.load()
    layer.E, layer.D, layer.k, layer.renorm = E, D, 4, 1
    wr = rng.normal(0, 1 / np.sqrt(D), size=(E, D)).astype(np.float32)
    bias = rng.normal(scale=0.1, size=E).astype(np.float32)
    layer.router_w = torch.from_numpy(wr).cuda()
    layer.router_bias = torch.from_numpy(bias).cuda()
    layer.sel_bias = None
    h = rng.normal(size=(T, D)).astype(np.float32)
    hd = torch.from_numpy(h).cuda()
    hb = torch.empty((T, D), dtype=torch.bfloat16, device='cuda')
    logits, ids, w = layer.route(hd, hb)
    ref = h.astype(np.float64) @ wr.T.astype(np.float64) + bias
    err = np.abs(logits.cpu().numpy().astype(np.float64) - ref).max() / np.abs(ref).max()
    assert err < 1e-6, err
    assert torch.equal(hb, hd.to(torch.bfloat16))


@pytest.mark.parametrize('T,E,k,D', [(16384, 64, 8, 4096), (1000, 16, 4, 512), (77, 8, 8, 8200)])
def test_scatter_equals_gather(T, E, k, D):
    """b200q_moe_scatter_bf16_dev (each token row read once, stored k times)
    fills the same rows as b200q_moe_gather_bf16_dev, bit for bit; D = 8200
    exercises the partial last chunk of the row loop."""
    from localai_b200 import _lib
    rng = np.random.default_rng(T + k)
    layer = QuantMoE.__new__(QuantMoE)
    layer.lib = _lib.load()
    layer.E, layer.D, layer.k = E, D, k
    ids = torch.from_numpy(np.argsort(rng.random((T, E)), axis=1)[:, :k].astype(np.int32)).cuda()
    w = torch.rand((T, k), device='cuda')
    hb = torch.randn((T, D), device='cuda').to(torch.bfloat16)
    offsets, slot_of, token_of, slot_w, _ = layer.dispatch(hb, ids, w, gather=False)
    a = layer.gather_bf16(hb, token_of)
    b = layer.scatter_bf16(hb, slot_of, token_of.numel())
    torch.cuda.synchronize()
    n = int(offsets[-1])
    assert n == T * k
    assert torch.equal(a[:n], b[:n])
    assert layer.lib.b200q_check_device_error() == 0


def test_router_logits_and_dispatch():
    rng = np.random.default_rng(3)
    E, D, F, k, T = 16, 512, 128, 4, 1000
    bias = np.log(np.arange(1, E + 1, dtype=np.float64) ** -1.1 / np.sum(np.arange(1, E + 1) ** -1.1)).astype(np.float32)
    layer, wr, *_ = make_layer(rng, E, D, F, k, router_bias=bias)
    h = rng.normal(size=(T, D)).astype(np.float32)
    hd = torch.from_numpy(h).cuda()
    logits, ids, w = layer.route(hd)
    ref = h.astype(np.float64) @ wr.T.astype(np.float64) + bias
    assert np.max(np.abs(logits.cpu().numpy() - ref)) / np.max(np.abs(ref)) < 1e-5
    offsets, slot_of, token_of, slot_w, xperm = layer.dispatch(hd, ids, w)
    torch.cuda.synchronize()
    ids_n, off, so, to = ids.cpu().numpy(), offsets.cpu().numpy(), slot_of.cpu().numpy(), token_of.cpu().numpy()
    counts = np.bincount(ids_n.reshape(-1), minlength=E)
    assert np.array_equal(off, np.concatenate([[0], np.cumsum(counts)]))
    # every (token, j) owns one slot inside its expert's range, in token order
    for e in range(E):
        seg = to[off[e]:off[e + 1]]
        assert np.all(np.diff(seg) > 0)
    flat_e = ids_n.reshape(-1)
    assert np.all((so >= off[flat_e]) & (so < off[flat_e + 1]))
    assert np.array_equal(to[so], np.repeat(np.arange(T), k))
    np.testing.assert_array_equal(slot_w.cpu().numpy()[so], w.cpu().numpy().reshape(-1))
    np.testing.assert_array_equal(xperm.float().cpu().numpy(), hd.to(torch.bfloat16).float().cpu().numpy()[to])


@pytest.mark.parametrize('E,D,F,k,T', [(8, 512, 128, 2, 300), (16, 1024, 192, 4, 600), (32, 512, 64, 8, 257)])
def test_layer_matches_oracle(E, D, F, k, T):
    rng = np.random.default_rng(E + D + F + k + T)
    layer, wr, gate_up, down, F_pad = make_layer(rng, E, D, F, k)
    h = rng.normal(size=(T, D)).astype(np.float32)
    y = layer(torch.from_numpy(h).cuda())
    torch.cuda.synchronize()
    from localai_b200 import ops
    ops.check_device_error()
    logits, ids, w = layer.route(torch.from_numpy(h).cuda())
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    # the top-k kernel is bit-exact on the GPU's own logits
    assert np.array_equal(ids, o.route_topk(logits.cpu().numpy(), k)[0])
    # against float64 logits the GPU's selected set may differ only where the
    # oracle's k-th and (k+1)-th probabilities are within ROUTE_MARGIN
    lg64 = h.astype(np.float64) @ wr.T.astype(np.float64)
    p64 = np.exp(lg64 - lg64.max(axis=1, keepdims=True))
    p64 /= p64.sum(axis=1, keepdims=True)
    order = np.argsort(-p64, axis=1, kind='stable')
    differ = np.nonzero(np.any(np.sort(ids, 1) != np.sort(order[:, :k], 1), axis=1))[0]
    if k < E:
        margin = p64[differ, order[differ, k - 1]] - p64[differ, order[differ, k]]
        assert np.all(margin <= ROUTE_MARGIN), (differ, margin)
    else:
        assert differ.size == 0
    experts = [(gate_up[e], down[e]) for e in range(E)]
    ref = o.moe_forward_f64(h, ids, w, experts, 12, 12, D, F, F_pad)
    assert o.normwise_rel_err(y.cpu().numpy(), ref) < 1e-2


@pytest.mark.parametrize('t_gu,t_dn', [(12, 14), (8, 12)])
@pytest.mark.parametrize('T', [2, 300])
def test_mixed_expert_types(t_gu, t_dn, T):
    """Gate/up and down experts of different GGML types (a Q6_K down beside
    Q4_K gate/up, as mixed quantisations store them; Q8_0 gate/up with Q4_K
    down): the decode-sized grouped-GEMV path (T = 2, f32 accumulation, 1e-3)
    and the tensor-core path (T = 300, bf16 operands, 1e-2) against the
    float64 oracle with the GPU's routing."""
    rng = np.random.default_rng(100 * t_gu + t_dn + T)
    E, D, F, k = 8, 512, 256, 2
    gate_up = [synth.make(rng, t_gu, 2 * F, D) for _ in range(E)]
    down = [synth.make(rng, t_dn, D, F) for _ in range(E)]
    wr = rng.normal(0, 1 / np.sqrt(D), size=(E, D)).astype(np.float32)
    cat = lambda parts: torch.frombuffer(bytearray(b''.join(parts)), dtype=torch.uint8).cuda()
    layer = QuantMoE(torch.from_numpy(wr).cuda(), cat(gate_up), cat(down), d_model=D, d_ff=F, top_k=k,
                     ggml_type=t_gu, down_type=t_dn)
    assert (T * k <= layer.small_slots) == (T == 2)
    h = rng.normal(size=(T, D)).astype(np.float32)
    y = layer(torch.from_numpy(h).cuda())
    _, ids, w = layer.route(torch.from_numpy(h).cuda())
    torch.cuda.synchronize()
    from localai_b200 import ops
    ops.check_device_error()
    ref = o.moe_forward_f64(h, ids.cpu().numpy(), w.cpu().numpy(), list(zip(gate_up, down)), t_gu, t_dn, D, F, F)
    assert o.normwise_rel_err(y.cpu().numpy(), ref) < (1e-3 if T == 2 else 1e-2)


def test_layer_deterministic():
    rng = np.random.default_rng(5)
    layer, *_ = make_layer(rng, 16, 512, 128, 4)
    h = torch.from_numpy(rng.normal(size=(333, 512)).astype(np.float32)).cuda()
    a = layer(h)
    b = layer(h)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize('chunks', [1, 3])
def test_forward_host_equals_chunked_forward(chunks):
    """forward_host (copies overlapped with compute) gives exactly forward()
    of each token chunk."""
    rng = np.random.default_rng(11)
    E, D, F, k, T = 16, 512, 128, 4, 301
    layer, *_ = make_layer(rng, E, D, F, k)
    h = torch.from_numpy(rng.normal(size=(T, D)).astype(np.float32)).pin_memory()
    y = layer.forward_host(h, chunks=chunks)
    torch.cuda.synchronize()
    bounds = chunk_bounds(T, chunks)
    ref = torch.cat([layer(h[a:b].cuda()).cpu() for a, b in zip(bounds[:-1], bounds[1:])])
    assert torch.equal(y, ref)
