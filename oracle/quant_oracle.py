"""CPU oracle for the GGML block-quant matvec/matmul and the MoE FFN.

TEST INFRASTRUCTURE ONLY.  This module restates, in NumPy, the reference
engine's algorithms for the accelerated path so that the CUDA library can be
checked against them.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or the timed CPU baseline -- never as the product path.

What each function restates (paths are relative to the reference project):

* ``LAYOUT`` / ``block_layout``        engine/dequant.py:6-17
* ``dequantize``                       engine/dequant.py:27-167 (NumPy branch);
  the numba branch (engine/numba_kernels.py:49-106) gives the same f32 bits.
* ``matvec_f64`` / ``matmul_f64``      the numeric oracle of the GEMV and MoE
  paths: ``dequantize(raw) @ x`` evaluated in float64.
* ``silu``                             engine/zaya.py:305 / engine/model.py:232
* ``route_topk``                       engine/zaya.py:290-296 generalised to
  top-k (stable: larger value first, lower index wins ties, as np.argmax).
* ``moe_forward_f64``                  engine/zaya.py:303-306 per token, summed
  over the k selected experts with the routing weights.
* ``rmsnorm_f32``                      engine/model.py:82
* ``gelu_exact``                       engine/zaya.py:181-186 (erf evaluated in
  float64 per element, result rounded to f32)
* ``zaya_router_f32``                  engine/zaya.py:278-296 router chain:
  projection, EDA term, RMSNorm, two GELU layers, logits over E+1 routes,
  softmax, top-1 over probs + route biases (first index on ties), weight =
  the unbiased probability
* ``llama_decode_f64``                 engine/model.py:174-240 (LlamaModel.forward,
  arch 'llama', no RoPE scaling): token by token with a KV cache, adjacent-
  pair RoPE, grouped-query attention, SiLU FFN, in float64
* ``zaya_moe_f64``                     engine/zaya.py:297-307: the selected
  expert's FFN (or, for the skip route E, the block input) times its weight

Rounding contract (bit-exact dequant): every product in the reference
formulas is exact in f32 (fp16 ``d`` has 11 significant bits; 6-bit scales and
4/5/6/8-bit quants keep every product within 24 bits), so the only rounding
is the single f32 subtraction of the Q4_K/Q5_K minimum term.
"""
from __future__ import annotations

import ctypes
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

# (values per block, bytes per block) -- engine/dequant.py:6-9
LAYOUT = {
    0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24),
    8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210),
}
Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 8, 12, 13, 14
MATVEC_TYPES = (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K)   # engine/native_quant.py:104


def block_layout(t):
    """engine/dequant.py:12-17."""
    if t not in LAYOUT:
        raise NotImplementedError(f'unsupported tensor type {t}')
    return LAYOUT[t]


def row_bytes(t, cols):
    block, nbytes = block_layout(t)
    if cols % block:
        raise ValueError(f'{cols} columns not divisible by block {block}')
    return (cols // block) * nbytes


def _half(blocks, offset):
    """fp16 field at byte ``offset`` of every block, widened exactly to f32."""
    lo = blocks[:, offset].astype(np.uint16)
    hi = blocks[:, offset + 1].astype(np.uint16)
    return (lo | (hi << 8)).view(np.float16).astype(np.float32)


def k_scales(scales):
    """Six-bit (scale, min) pairs of a Q4_K/Q5_K super-block.

    engine/dequant.py:108-113: sub-block g<4 reads the low 6 bits of s[g] and
    s[g+4]; g>=4 combines a nibble of s[g+4] with the top two bits of s[g-4]
    (scale) or s[g] (min).  Returns two uint8 arrays of shape [blocks, 8].
    """
    s = scales.astype(np.uint8)
    sc = np.empty((s.shape[0], 8), np.uint8)
    mn = np.empty((s.shape[0], 8), np.uint8)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def _affine_k(q, d, dmin, sc, mn):
    """fl(q * fl(d*sc)) - fl(dmin*mn) in f32 (engine/dequant.py:117-120)."""
    step = (d[:, None] * sc.astype(np.float32))            # [blocks, 8], exact
    low = (dmin[:, None] * mn.astype(np.float32))           # [blocks, 8], exact
    qf = q.astype(np.float32).reshape(q.shape[0], 8, 32)
    return (qf * step[:, :, None] - low[:, :, None]).reshape(q.shape[0], 256)


def _q4_k(blocks):
    d, dmin = _half(blocks, 0), _half(blocks, 2)
    sc, mn = k_scales(blocks[:, 4:16])
    qs = blocks[:, 16:144].reshape(-1, 4, 32)
    # 32-byte chunk p: low nibbles -> sub-block 2p, high nibbles -> 2p+1.
    q = np.stack((qs & 15, qs >> 4), axis=2).reshape(-1, 256)
    return _affine_k(q, d, dmin, sc, mn)


def _q5_k(blocks):
    d, dmin = _half(blocks, 0), _half(blocks, 2)
    sc, mn = k_scales(blocks[:, 4:16])
    qh = blocks[:, 16:48]                                   # [blocks, 32]
    qs = blocks[:, 48:176].reshape(-1, 4, 32)
    low = np.stack((qs & 15, qs >> 4), axis=2).reshape(-1, 8, 32)
    high = (qh[:, None, :] >> np.arange(8, dtype=np.uint8)[None, :, None]) & 1
    q = (low | (high << 4)).reshape(-1, 256)
    return _affine_k(q, d, dmin, sc, mn)


def _q6_k(blocks):
    ql = blocks[:, 0:128].reshape(-1, 2, 2, 32)             # [b, half, lo/hi 32, j]
    qh = blocks[:, 128:192].reshape(-1, 2, 32)              # [b, half, j]
    sc = blocks[:, 192:208].view(np.int8).reshape(-1, 2, 4, 2)  # [b, half, quad, j//16]
    d = _half(blocks, 208)
    out = np.empty((blocks.shape[0], 2, 4, 32), np.float32)
    for quad in range(4):
        nib = ql[:, :, quad & 1, :]
        nib = (nib & 15) if quad < 2 else (nib >> 4)
        q = nib | (((qh >> (2 * quad)) & 3) << 4)
        s = np.repeat(sc[:, :, quad, :], 16, axis=2).astype(np.float32)
        # engine/dequant.py:165 -- ((q-32) * d) * scale, all exact in f32
        out[:, :, quad, :] = (q.astype(np.int16) - 32).astype(np.float32) * d[:, None, None] * s
    return out.reshape(-1, 256)


def _q8_0(blocks):
    d = _half(blocks, 0)
    return blocks[:, 2:34].view(np.int8).astype(np.float32) * d[:, None]


def _q4_0(blocks):
    d = _half(blocks, 0)
    qs = blocks[:, 2:18]
    q = np.concatenate((qs & 15, qs >> 4), axis=1).astype(np.float32) - 8.0
    return q * d[:, None]


def _q4_1(blocks):
    d, m = _half(blocks, 0), _half(blocks, 2)
    qs = blocks[:, 4:20]
    q = np.concatenate((qs & 15, qs >> 4), axis=1).astype(np.float32)
    return q * d[:, None] + m[:, None]


def _q5_x(blocks, with_min):
    d = _half(blocks, 0)
    m = _half(blocks, 2) if with_min else None
    off = 4 if with_min else 2
    qh = blocks[:, off:off + 4]
    qs = blocks[:, off + 4:off + 20]
    low = np.concatenate((qs & 15, qs >> 4), axis=1).astype(np.int16)
    bit = np.arange(32)
    high = ((qh[:, bit // 8] >> (bit % 8).astype(np.uint8)) & 1).astype(np.int16)
    q = low | (high << 4)
    if with_min:
        return q.astype(np.float32) * d[:, None] + m[:, None]
    return (q.astype(np.float32) - 16.0) * d[:, None]


_DECODERS = {Q4_0: _q4_0, 3: _q4_1, 6: lambda b: _q5_x(b, False),
             7: lambda b: _q5_x(b, True), Q8_0: _q8_0, Q4_K: _q4_k,
             Q5_K: _q5_k, Q6_K: _q6_k}


def dequantize(raw, t, shape):
    """Decode packed GGML blocks to f32 -- engine/dequant.py:27-167."""
    block, nbytes = block_layout(t)
    n = int(np.prod(shape, dtype=np.int64))
    if n % block:
        raise ValueError(f'{n} elements is not divisible by block size {block}')
    if t == 0:
        return np.frombuffer(raw, dtype='<f4', count=n).copy().reshape(shape)
    if t == 1:
        return np.frombuffer(raw, dtype='<f2', count=n).astype(np.float32).reshape(shape)
    blocks = np.frombuffer(raw, dtype=np.uint8, count=(n // block) * nbytes)
    blocks = blocks.reshape(n // block, nbytes)
    return _DECODERS[t](blocks).reshape(shape)


_C_ORACLE = None


def _c_oracle():
    """The C restatement (oracle/quant_oracle.c, built by ``make -C oracle``),
    or None when it is not built.  tests/test_oracle.py checks that its decode
    equals ``dequantize`` bit for bit."""
    global _C_ORACLE
    if _C_ORACLE is None:
        so = Path(__file__).resolve().parent / '_build' / 'liboracle.so'
        _C_ORACLE = ctypes.CDLL(str(so)) if so.exists() else False
    return _C_ORACLE or None


def dequantize_fast(raw, t, shape):
    """``dequantize`` through the C restatement when it is built (same f32
    bits, several times faster on large matrices; releases the GIL), else the
    NumPy restatement."""
    lib = _c_oracle()
    if lib is None or t not in MATVEC_TYPES:
        return dequantize(raw, t, shape)
    block, nbytes = block_layout(t)
    n = int(np.prod(shape, dtype=np.int64))
    if n % block:
        raise ValueError(f'{n} elements is not divisible by block size {block}')
    buf = np.frombuffer(raw, dtype=np.uint8, count=(n // block) * nbytes)
    out = np.empty(n, np.float32)
    if lib.oracle_dequant(t, buf.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                          ctypes.c_longlong(n // block)) != 0:
        raise ValueError(f'C oracle cannot decode type {t}')
    return out.reshape(shape)


def matvec_f64(raw, t, rows, cols, x):
    """``dequantize(raw) @ x`` in float64: the GEMV parity oracle."""
    w = dequantize_fast(raw, t, (rows, cols)).astype(np.float64)
    return w @ np.asarray(x, np.float64)


def matmul_f64(raw, t, rows, cols, vectors):
    """[tokens, cols] x W[rows, cols]^T in float64 -> [tokens, rows]."""
    w = dequantize_fast(raw, t, (rows, cols)).astype(np.float64)
    return np.asarray(vectors, np.float64) @ w.T


def normwise_rel_err(got, ref):
    """max|got-ref| / max|ref| -- the tolerance metric for GEMV/MoE outputs."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = float(np.max(np.abs(ref))) if ref.size else 0.0
    return float(np.max(np.abs(got - ref))) / max(denom, 1e-300) if ref.size else 0.0


def silu(g):
    """engine/zaya.py:305 -- g / (1 + exp(-clip(g, -80, 80)))."""
    g = np.asarray(g)
    return g / (1.0 + np.exp(-np.clip(g, -80, 80)))


def softmax_f32(logits):
    """engine/zaya.py:290 -- max-subtracted softmax, every step in f32, per row."""
    z = np.asarray(logits, np.float32)
    z = z - z.max(axis=-1, keepdims=True)
    p = np.exp(z)
    return p / p.sum(axis=-1, keepdims=True)


def route_topk(logits, k, bias=None, renormalize=True):
    """Softmax -> optional additive selection bias -> stable top-k -> weights.

    engine/zaya.py:290-296 is the k=1 case (argmax of ``probs + bias``, weight
    = unbiased ``probs[e]``, not renormalised).  Ties go to the lower expert
    index, as ``np.argmax`` does.  Returns (ids int32 [T,k], weights f32 [T,k]).
    With ``renormalize`` the weights are ``p_i / sum_topk p`` computed in f32
    by a left-to-right sum over the k selected probabilities.
    """
    probs = softmax_f32(np.atleast_2d(logits))
    sel = probs if bias is None else (probs + np.asarray(bias, np.float32)).astype(np.float32)
    # stable descending sort: lexsort on (index, -value)
    order = np.argsort(-sel, axis=-1, kind='stable')[:, :k].astype(np.int32)
    w = np.take_along_axis(probs, order, axis=-1).astype(np.float32)
    if renormalize:
        total = np.zeros(w.shape[0], np.float32)
        for j in range(k):
            total = (total + w[:, j]).astype(np.float32)
        w = (w / total[:, None]).astype(np.float32)
    return order, w


def expert_ffn_f64(gate_up_raw, down_raw, t_gu, t_dn, d_model, d_ff, d_ff_padded, h):
    """One expert on a batch: down(silu(gate h) * up h) -- engine/zaya.py:303-306.

    ``gate_up_raw`` is the packed [2F, D] matrix (gate rows first, then up
    rows, as np.split(packed, 2) reads them); ``down_raw`` is [D, F_padded].
    Returns float64 [tokens, D].
    """
    h = np.atleast_2d(np.asarray(h, np.float64))
    gu = matmul_f64(gate_up_raw, t_gu, 2 * d_ff, d_model, h)
    gate, up = gu[:, :d_ff], gu[:, d_ff:]
    act = np.zeros((h.shape[0], d_ff_padded), np.float64)
    act[:, :d_ff] = silu(gate) * up
    return matmul_f64(down_raw, t_dn, d_model, d_ff_padded, act)


def moe_forward_f64(h, ids, weights, experts, t_gu, t_dn, d_model, d_ff, d_ff_padded, workers=1):
    """Weighted combine over the selected experts.

    ``experts[e] = (gate_up_raw, down_raw)`` (a list, dict or callable).
    Tokens are grouped per expert (each expert's product runs once over its
    tokens), then ``y[t] = sum_j w[t,j] * out_e(t)``.  ``workers`` > 1 runs the
    experts' products in threads; the sum is still taken in expert order.
    """
    h = np.atleast_2d(np.asarray(h, np.float32))
    T, k = ids.shape
    y = np.zeros((T, d_model), np.float64)
    get = experts if callable(experts) else experts.__getitem__

    def one(e):
        # a token selects an expert at most once, so ``rows`` is duplicate-free
        rows, slots = np.nonzero(ids == e)
        gu, dn = get(int(e))
        return rows, slots, expert_ffn_f64(gu, dn, t_gu, t_dn, d_model, d_ff, d_ff_padded, h[rows])

    uniq = np.unique(ids)
    if workers > 1:
        with ThreadPoolExecutor(max_workers=workers) as ex:
            results = list(ex.map(one, uniq))
    else:
        results = [one(e) for e in uniq]
    for rows, slots, out in results:
        y[rows] += out * weights[rows, slots].astype(np.float64)[:, None]
    return y


def rmsnorm_f32(x, w, eps):
    """x * (1 / sqrt(mean(x * x) + eps)) * w, f32 (engine/model.py:82)."""
    x = np.asarray(x, np.float32)
    return x * (np.float32(1.0) / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + np.float32(eps))) * w


def gelu_exact(x):
    """Exact GELU, erf in float64 per element (engine/zaya.py:181-186)."""
    import math
    flat = np.asarray(x, np.float32).reshape(-1)
    out = np.fromiter((v * (1.0 + math.erf(float(v) / math.sqrt(2.0))) * 0.5 for v in flat),
                      dtype=np.float32, count=flat.size)
    return out.reshape(np.shape(x))


def _linear_f32(x, w, b=None):
    y = (np.asarray(x, np.float32) @ np.asarray(w, np.float32).T).astype(np.float32)
    return y if b is None else (y + b).astype(np.float32)


def zaya_router_f32(h, w_in, w_gate, w_mlp2, w_mlp4, norm_w, biases, eps, prev=None, w_eda=None,
                    b_in=None, b_gate=None, b_mlp2=None, b_mlp4=None):
    """Batched restatement of the router chain of engine/zaya.py:278-296.

    Returns (expert [T], weight [T], probs [T, E+1], router_state [T, R]);
    expert == E is the learned skip route.
    """
    r = _linear_f32(h, w_in, b_in)
    if prev is not None and w_eda is not None:
        r = (r + prev * w_eda).astype(np.float32)
    state = r.copy()
    r = rmsnorm_f32(r, norm_w, eps)
    r = gelu_exact(_linear_f32(r, w_gate, b_gate))
    r = gelu_exact(_linear_f32(r, w_mlp2, b_mlp2))
    logits = _linear_f32(r, w_mlp4, b_mlp4)
    logits = logits - logits.max(axis=-1, keepdims=True)
    probs = np.exp(logits)
    probs = (probs / probs.sum(axis=-1, keepdims=True)).astype(np.float32)
    route = probs + biases
    expert = np.argmax(route, axis=-1)
    weight = probs[np.arange(len(expert)), expert]
    return expert, weight, probs, state


def zaya_moe_f64(h, expert, weight, experts, t_gu, t_dn, d_model, d_ff, d_ff_padded):
    """engine/zaya.py:297-307 for a batch: y[t] = w[t] * FFN_e(h[t]), or
    w[t] * h[t] for the skip route e == len(experts)."""
    h = np.atleast_2d(np.asarray(h, np.float32))
    E = len(experts)
    y = np.zeros(h.shape, np.float64)
    for e in np.unique(expert):
        rows = np.nonzero(expert == e)[0]
        if e == E:
            out = h[rows].astype(np.float64)
        else:
            out = expert_ffn_f64(experts[e][0], experts[e][1], t_gu, t_dn, d_model, d_ff, d_ff_padded, h[rows])
        y[rows] = out * weight[rows].astype(np.float64)[:, None]
    return y


def rope_inv_f64(cfg, half):
    """Per-pair RoPE frequencies in float64 (engine/model.py:199-214): plain
    base^(-j/half); 'llama3' keeps wavelengths below orig/high, divides those
    above orig/low by the factor and blends linearly in between; 'linear'
    divides by the factor (the reference divides the angle, the same up to
    rounding)."""
    inv = 1.0 / (cfg['rope_base'] ** (np.arange(half, dtype=np.float64) / max(half, 1)))
    kind = str(cfg.get('rope_scaling', 'none')).lower()
    fac = float(cfg.get('rope_factor', 1.0))
    if kind == 'none' or fac <= 1.0:
        return inv
    if kind == 'linear':
        return inv / fac
    orig = float(cfg.get('rope_orig_ctx', 8192))
    lo, hi = float(cfg.get('rope_low_freq', 1.0)), float(cfg.get('rope_high_freq', 4.0))
    wl = 2.0 * np.pi / inv
    smooth = (orig / wl - lo) / (hi - lo)
    mid = (1.0 - smooth) * inv / fac + smooth * inv
    return np.where(wl > orig / lo, inv / fac, np.where(wl < orig / hi, inv, mid))


def llama_decode_f64(w, cfg, tokens):
    """Logits after each token of ``tokens`` (positions 0, 1, ...), float64.

    ``w``: {'token_embd': [V, D], 'output': [V, D], 'output_norm': [D],
    'layers': [{'attn_q': [H*hd, D], 'attn_k': [KV*hd, D], 'attn_v',
    'attn_output': [D, D], 'ffn_gate': [F, D], 'ffn_up', 'ffn_down': [D, F],
    'attn_norm': [D], 'ffn_norm': [D]}]} as float arrays; ``cfg`` with
    n_heads, n_kv_heads, rope_base, eps (and optional rope_dim, and RoPE
    scaling: rope_scaling 'llama3' / 'linear' with rope_factor, rope_orig_ctx,
    rope_low_freq, rope_high_freq -- engine/model.py:199-214; arch 'qwen2' /
    'qwen3': split-half RoPE pairs, engine/model.py:212-221).  A layer may add
    'attn_q_bias' / 'attn_k_bias' / 'attn_v_bias' (projection biases,
    engine/model.py:73-79) and 'attn_q_norm' / 'attn_k_norm' (per-head RMSNorm
    weights [hd], engine/model.py:188-192); cfg 'sliding_window' > 0 limits
    attention to the last that many positions (engine/model.py:222).
    """
    H, KV = cfg['n_heads'], cfg['n_kv_heads']
    D = w['token_embd'].shape[1]
    hd = D // H
    rotary = min(cfg.get('rope_dim') or hd, hd)
    rotary -= rotary % 2
    half = rotary // 2
    eps = cfg['eps']
    norm = lambda x, g: x * (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)) * g
    neox = cfg.get('arch', 'llama') != 'llama'
    nl = len(w['layers'])
    kc = [[] for _ in range(nl)]
    vc = [[] for _ in range(nl)]
    out = []
    for pos, tok in enumerate(tokens):
        x = w['token_embd'][tok].astype(np.float64)
        inv = rope_inv_f64(cfg, half)
        ang = pos * inv
        c, s_ = np.cos(ang), np.sin(ang)

        def rope(a):
            z = a.copy()
            if neox:
                e, o = a[:, :half].copy(), a[:, half:rotary].copy()
                z[:, :half] = e * c - o * s_
                z[:, half:rotary] = e * s_ + o * c
            else:
                e, o = a[:, 0:rotary:2].copy(), a[:, 1:rotary:2].copy()
                z[:, 0:rotary:2] = e * c - o * s_
                z[:, 1:rotary:2] = e * s_ + o * c
            return z

        def proj(L, name, h, heads):
            y = L[name] @ h
            if name + '_bias' in L:
                y = y + L[name + '_bias']
            y = y.reshape(heads, hd)
            if name + '_norm' in L:
                y = norm(y, L[name + '_norm'])
            return y
        for li, L in enumerate(w['layers']):
            pre = x
            h = norm(x, L['attn_norm'])
            q = rope(proj(L, 'attn_q', h, H))
            k = rope(proj(L, 'attn_k', h, KV))
            v = proj(L, 'attn_v', h, KV)
            kc[li].append(k)
            vc[li].append(v)
            w0 = max(0, pos + 1 - cfg['sliding_window']) if cfg.get('sliding_window', 0) > 0 else 0
            ks, vs = np.stack(kc[li][w0:]), np.stack(vc[li][w0:])   # [L, KV, hd] (engine/model.py:222)
            g = H // KV
            att = np.empty((H, hd))
            for hh in range(H):
                sc = ks[:, hh // g, :] @ q[hh] / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                p /= p.sum()
                att[hh] = p @ vs[:, hh // g, :]
            x = pre + L['attn_output'] @ att.reshape(-1)
            pre = x
            h = norm(x, L['ffn_norm'])
            gt, up = L['ffn_gate'] @ h, L['ffn_up'] @ h
            x = pre + L['ffn_down'] @ (gt / (1.0 + np.exp(-np.clip(gt, -80, 80))) * up)
        out.append(w['output'] @ norm(x, w['output_norm']))
    return np.stack(out)
