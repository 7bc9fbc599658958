"""CPU tests: pin the oracle to the reference before trusting it.

* golden fixtures produced by the reference's own engine/dequant.py
  (tests/golden/make_golden.py) -- bit-exact;
* the reference's known-answer byte patterns (tests/test_dequant.py:36-95 of
  the reference), restated here as test vectors;
* the C restatement (oracle/quant_oracle.c) against the NumPy one;
* the reference's own native library built from its source by
  oracle/Makefile (when present) against the oracle, with the reference
  test tolerances (tests/test_dequant.py:119-230).
"""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import quant_oracle as o
from localai_b200 import synth

ROOT = Path(__file__).resolve().parent.parent
ORACLE_SO = ROOT / 'oracle' / '_build' / 'liboracle.so'
REF_SO = ROOT / 'oracle' / '_ref' / 'libnative_quant_ref.so'


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_golden_bit_exact(golden):
    assert len(golden) >= 8
    for name, t, rows, cols, raw, ref in golden:
        got = o.dequantize(raw, t, (rows, cols))
        assert got.dtype == np.float32
        assert np.array_equal(bits(got), bits(ref)), name


# ---- known-answer vectors of the reference tests (tests/test_dequant.py:36-95)
def test_layouts():
    assert o.block_layout(0) == (1, 4) and o.block_layout(1) == (1, 2)
    assert o.block_layout(2) == (32, 18) and o.block_layout(3) == (32, 20)
    assert o.block_layout(6) == (32, 22) and o.block_layout(7) == (32, 24)
    assert o.block_layout(8) == (32, 34) and o.block_layout(12) == (256, 144)
    assert o.block_layout(13) == (256, 176) and o.block_layout(14) == (256, 210)
    with pytest.raises(NotImplementedError):
        o.block_layout(99)


def test_q8_0_arange():
    raw = np.float16(0.5).tobytes() + np.arange(-16, 16, dtype=np.int8).tobytes()
    np.testing.assert_array_equal(o.dequantize(raw, 8, (32,)), np.arange(-16, 16, dtype=np.float32) * .5)


def test_q4_0_and_q5_variants():
    raw = np.float16(1).tobytes() + bytes([0x98]) * 16
    out = o.dequantize(raw, 2, (32,))
    assert np.all(out[:16] == 0) and np.all(out[16:] == 1)
    raw = np.float16(1).tobytes() + bytes(4) + bytes([0x98]) * 16
    out = o.dequantize(raw, 6, (32,))
    assert np.all(out[:16] == -8) and np.all(out[16:] == -7)
    raw = np.float16(.5).tobytes() + np.float16(1).tobytes() + bytes(4) + bytes([0x21]) * 16
    out = o.dequantize(raw, 7, (32,))
    assert np.all(out[:16] == 1.5) and np.all(out[16:] == 2.0)
    raw = np.float16(.5).tobytes() + np.float16(1).tobytes() + bytes([0x21]) * 16
    out = o.dequantize(raw, 3, (32,))
    assert np.all(out[:16] == 1.5) and np.all(out[16:] == 2.0)


def test_q4_k_nibble_interleave_and_zero_block():
    scales = bytes([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])
    qs = bytes([0x10] * 32 + [0x20] * 32 + [0x30] * 32 + [0x40] * 32)
    raw = np.float16(1).tobytes() + np.float16(0).tobytes() + scales + qs
    out = o.dequantize(raw, 12, (256,))
    for g, e in enumerate((0, 1, 0, 2, 0, 3, 0, 4)):
        assert np.all(out[g * 32:(g + 1) * 32] == e)
    raw = np.float16(1).tobytes() + np.float16(0).tobytes() + bytes(140)
    assert np.all(o.dequantize(raw, 12, (256,)) == 0)
    qs = bytes([0x21]) * 128
    raw = np.float16(1).tobytes() + np.float16(0).tobytes() + scales + qs
    out = o.dequantize(raw, 12, (256,))
    for g in range(8):
        assert np.all(out[g * 32:(g + 1) * 32] == (1 if g % 2 == 0 else 2))


def test_q5_k_high_bit_planes():
    scales = bytes([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])
    qs = bytes([0x10] * 32 + [0x20] * 32 + [0x30] * 32 + [0x40] * 32)
    raw = np.float16(1).tobytes() + np.float16(0).tobytes() + scales + bytes([0xFF]) * 32 + qs
    out = o.dequantize(raw, 13, (256,))
    for g, e in enumerate((16, 17, 16, 18, 16, 19, 16, 20)):
        assert np.all(out[g * 32:(g + 1) * 32] == e)


def test_q6_k_zero_and_packed_quads():
    raw = bytes(128 + 64 + 16) + np.float16(1).tobytes()
    assert np.all(o.dequantize(raw, 14, (256,)) == 0)
    raw = bytes([0x98]) * 128 + bytes(64) + np.ones(16, np.int8).tobytes() + np.float16(1).tobytes()
    out = o.dequantize(raw, 14, (256,))
    assert np.all(out[:64] == -24) and np.all(out[64:128] == -23)
    assert np.all(out[128:192] == -24) and np.all(out[192:] == -23)


# ---- synthetic generators produce what they claim
def test_k_scale_packing_roundtrip():
    rng = np.random.default_rng(3)
    sc = rng.integers(0, 64, size=(50, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(50, 8), dtype=np.uint8)
    s = synth.pack_k_scales(sc, mn)
    got_sc, got_mn = o.k_scales(s)
    assert np.array_equal(got_sc, sc) and np.array_equal(got_mn, mn)


def test_q4k_padding_decodes_to_zero():
    rng = np.random.default_rng(4)
    raw = synth.q4_k(rng, 5, 1536, zero_tail_cols=128)
    w = o.dequantize(raw, 12, (5, 1536))
    assert np.all(w[:, 1408:] == 0) and np.any(w[:, :1408] != 0)


# ---- routing oracle properties (engine/zaya.py:290-296 generalised)
def test_route_topk_k1_is_zaya_argmax():
    rng = np.random.default_rng(5)
    logits = rng.normal(size=(64, 17)).astype(np.float32)
    bias = rng.normal(scale=0.1, size=17).astype(np.float32)
    ids, w = o.route_topk(logits, 1, bias=bias, renormalize=False)
    for t in range(64):
        z = logits[t] - logits[t].max()
        p = np.exp(z)
        p /= p.sum()
        e = int(np.argmax(p + bias))
        assert ids[t, 0] == e and w[t, 0] == p[e]


def test_route_topk_ties_prefer_lower_index():
    logits = np.zeros((1, 8), np.float32)
    ids, w = o.route_topk(logits, 3)
    assert ids.tolist() == [[0, 1, 2]]
    np.testing.assert_allclose(w, 1 / 3, rtol=1e-6)


def test_silu_clip():
    g = np.array([-100.0, -1.0, 0.0, 1.0, 100.0], np.float32)
    np.testing.assert_allclose(o.silu(g), g / (1 + np.exp(-np.clip(g, -80, 80))))


# ---- C restatement and the reference's own library
def _build_oracle_so():
    if not ORACLE_SO.exists():
        subprocess.run(['make', '-C', str(ROOT / 'oracle'), 'all'], check=True, capture_output=True)
    return ctypes.CDLL(str(ORACLE_SO))


def test_c_oracle_matches_numpy_oracle(golden):
    lib = _build_oracle_so()
    for name, t, rows, cols, raw, ref in golden:
        if t not in o.MATVEC_TYPES:
            continue
        nblocks = rows * cols // o.block_layout(t)[0]
        out = np.empty(rows * cols, np.float32)
        buf = np.frombuffer(raw, np.uint8)
        assert lib.oracle_dequant(t, buf.ctypes.data_as(ctypes.c_void_p),
                                  out.ctypes.data_as(ctypes.c_void_p), ctypes.c_longlong(nblocks)) == 0
        assert np.array_equal(bits(out), bits(ref.reshape(-1))), name
        x = np.random.default_rng(1).normal(size=(3, cols)).astype(np.float32)
        y = np.empty((3, rows), np.float64)
        assert lib.oracle_matmul_f64(t, buf.ctypes.data_as(ctypes.c_void_p), x.ctypes.data_as(ctypes.c_void_p),
                                     y.ctypes.data_as(ctypes.c_void_p), rows, cols, 3) == 0
        np.testing.assert_allclose(y, o.matmul_f64(raw, t, rows, cols, x), rtol=1e-12, atol=1e-12)


def _ref_lib():
    if not REF_SO.exists():
        pytest.skip('reference library not built (make -C oracle ref needs the reference checkout)')
    lib = ctypes.CDLL(str(REF_SO))
    return lib


@pytest.mark.parametrize('t,seed,rtol,atol', [(8, 50, 2e-5, 2e-4), (14, 52, 2e-4, 2e-3), (2, 55, 2e-4, 2e-3)])
def test_reference_library_matches_oracle(t, seed, rtol, atol):
    """The compiled reference kernels agree with the oracle where the
    reference's own tests say they do (tests/test_dequant.py:119-144,218-230)."""
    lib = _ref_lib()
    rng = np.random.default_rng(seed)
    rows, cols = 300, 512
    raw = synth.random_blocks(rng, t, rows, cols, d=0.03125 if t != 14 else 0.0005)
    x = rng.normal(size=cols).astype(np.float32)
    out = np.empty(rows, np.float32)
    name = {8: 'localai_q8_0_matvec', 14: 'localai_q6k_matvec', 2: 'localai_q4_0_matvec'}[t]
    buf = np.frombuffer(raw, np.uint8)
    getattr(lib, name)(buf.ctypes.data_as(ctypes.c_void_p), x.ctypes.data_as(ctypes.c_void_p),
                       out.ctypes.data_as(ctypes.c_void_p), rows, cols, 4)
    np.testing.assert_allclose(out, o.dequantize(raw, t, (rows, cols)) @ x, rtol=rtol, atol=atol)


def test_reference_q4k_is_approximate():
    """The reference Q4_K kernel quantises x to int8 (engine/native_quant.cpp:84-109):
    against the exact product its normwise error is far above 1e-3 -- which is
    why parity is measured against dequantize(raw) @ x and not against it."""
    lib = _ref_lib()
    rng = np.random.default_rng(7)
    rows, cols = 512, 4096
    raw = synth.q4_k(rng, rows, cols)
    x = rng.normal(size=cols).astype(np.float32)
    out = np.empty(rows, np.float32)
    buf = np.frombuffer(raw, np.uint8)
    lib.localai_q4k_matvec(buf.ctypes.data_as(ctypes.c_void_p), x.ctypes.data_as(ctypes.c_void_p),
                           out.ctypes.data_as(ctypes.c_void_p), rows, cols, 4)
    err = o.normwise_rel_err(out, o.matvec_f64(raw, 12, rows, cols, x))
    assert 1e-3 < err < 5e-2


def test_zaya_router_oracle_matches_reference_golden():
    """The batched router-chain restatement reproduces the reference's own
    ZayaModel._moe (engine/zaya.py:274-307) on the committed fixture: same
    routes (skip route included), router state and block output to f32
    accuracy (the fixture's experts are f32 matrices)."""
    d = np.load(Path(__file__).resolve().parent / 'golden' / 'zaya_moe_golden.npz')
    H, P = d['H'], d['P']
    T = H.shape[0]
    use_prev = (np.arange(T) % 3) != 0
    Pm = np.where(use_prev[:, None], P, 0.0).astype(np.float32)
    # rows without a previous router state: EDA term absent (zero prev is the same)
    e, w, probs, state = o.zaya_router_f32(H, d['ffn_gate_inp_weight'], d['ffn_gate_weight'],
                                           d['zaya_router_mlp2_weight'], d['zaya_router_mlp4_weight'],
                                           d['ffn_norm_weight'], d['zaya_router_biases_weight'], float(d['eps']),
                                           prev=Pm, w_eda=d['zaya_router_eda_weight'], b_in=d['b_in'])
    np.testing.assert_allclose(state, d['S'], rtol=1e-5, atol=1e-6)
    E = d['gu'].shape[0]
    y = np.zeros_like(H, dtype=np.float64)
    for t in range(T):
        if e[t] == E:
            y[t] = H[t] * w[t]
        else:
            g = d['gu'][e[t]] @ H[t]
            F = g.shape[0] // 2
            act = o.silu(g[:F]) * g[F:]
            y[t] = (d['dn'][e[t]] @ act) * w[t]
    ref_routes_skip = np.sum(e == E)
    assert ref_routes_skip > 0 and ref_routes_skip < T          # the fixture exercises both kinds
    assert o.normwise_rel_err(y, d['Y']) < 1e-5


def test_llama_decode_oracle_matches_reference_golden():
    """The float64 decoder restatement reproduces the reference's own
    LlamaModel.forward (engine/model.py:174-240) on the committed fixture:
    RoPE layout, grouped-query attention, norms and FFN (f32 weights)."""
    d = np.load(Path(__file__).resolve().parent / 'golden' / 'llama_decode_golden.npz')
    NL = 2
    w = {'token_embd': d['token_embd_weight'], 'output': d['output_weight'], 'output_norm': d['output_norm_weight'],
         'layers': [{n: d[f'blk_{l}_{n}_weight'] for n in ('attn_q', 'attn_k', 'attn_v', 'attn_output', 'ffn_gate',
                                                             'ffn_up', 'ffn_down', 'attn_norm', 'ffn_norm')}
                    for l in range(NL)]}
    cfg = {'n_heads': 4, 'n_kv_heads': 2, 'rope_base': 10000.0, 'eps': 1e-5}
    got = o.llama_decode_f64(w, cfg, list(d['tokens']))
    assert o.normwise_rel_err(got, d['logits'].astype(np.float64)) < 1e-5
    # RoPE scaling (engine/model.py:199-214): llama3 interpolation and linear
    for kind, fac in (('llama3', 8.0), ('linear', 4.0)):
        sc = dict(cfg, rope_scaling=kind, rope_factor=fac, rope_orig_ctx=64, rope_low_freq=1.0, rope_high_freq=4.0)
        got = o.llama_decode_f64(w, sc, list(d['tokens']))
        ref = d['logits_' + kind].astype(np.float64)
        assert o.normwise_rel_err(got, ref) < 1e-5, kind
        assert o.normwise_rel_err(ref, d['logits'].astype(np.float64)) > 1e-2     # the scaling changes the logits
    # Qwen layouts (engine/model.py:184-221): split-half RoPE pairs; qwen3 with
    # per-head q/k norms, qwen2 with q/k/v projection biases
    for arch in ('qwen3', 'qwen2'):
        lw = []
        for l in range(NL):
            L = dict(w['layers'][l])
            if arch == 'qwen3':
                L['attn_q_norm'] = d[f'blk_{l}_attn_q_norm_weight']
                L['attn_k_norm'] = d[f'blk_{l}_attn_k_norm_weight']
            else:
                for n in ('q', 'k', 'v'):
                    L[f'attn_{n}_bias'] = d[f'blk_{l}_attn_{n}_bias']
            lw.append(L)
        got = o.llama_decode_f64(dict(w, layers=lw), dict(cfg, arch=arch), list(d['tokens']))
        ref = d['logits_' + arch].astype(np.float64)
        assert o.normwise_rel_err(got, ref) < 1e-5, arch
        assert o.normwise_rel_err(ref, d['logits'].astype(np.float64)) > 1e-2
    # sliding window of 3 positions (engine/model.py:222)
    got = o.llama_decode_f64(w, dict(cfg, sliding_window=3), list(d['tokens']))
    assert o.normwise_rel_err(got, d['logits_window3'].astype(np.float64)) < 1e-5


def test_rope_frequency_table_matches_oracle():
    """localai_b200.decoder.rope_inv_freq (float32, uploaded for the RoPE
    kernel) against the oracle's float64 frequencies, all three llama3 bands
    and linear, within f32 rounding."""
    from localai_b200.decoder import LlamaConfig, rope_inv_freq
    for kind, fac, base, rot in (('llama3', 8.0, 500000.0, 128), ('llama3', 8.0, 10000.0, 16),
                                 ('linear', 4.0, 10000.0, 64)):
        c = LlamaConfig(n_layers=1, d_model=32 * rot, n_heads=32, n_kv_heads=8, d_ff=64, vocab=8, rope_base=base,
                        rope_scaling=kind, rope_factor=fac, rope_orig_ctx=64 if rot == 16 else 8192)
        got = rope_inv_freq(c, rot).astype(np.float64)
        ref = o.rope_inv_f64({'rope_base': base, 'rope_scaling': kind, 'rope_factor': fac,
                              'rope_orig_ctx': c.rope_orig_ctx, 'rope_low_freq': 1.0, 'rope_high_freq': 4.0}, rot // 2)
        np.testing.assert_allclose(got, ref, rtol=2e-6)
    plain = LlamaConfig(n_layers=1, d_model=64, n_heads=1, n_kv_heads=1, d_ff=64, vocab=8)
    assert rope_inv_freq(plain, 64) is None
