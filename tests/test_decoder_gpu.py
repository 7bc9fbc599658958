"""GPU tests of the greedy decode step (engine/model.py:174-240) against the
float64 decoder oracle (pinned to the reference's own LlamaModel.forward by
tests/golden/llama_decode_golden.npz).

Logits after every token: normwise <= 1e-3 (f32 accumulation throughout);
greedy tokens equal to the oracle's argmax; the CUDA-graph replay gives the
same logits as the eager step, bit for bit.
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import synth
from localai_b200.decoder import LlamaConfig, QuantLlama

pytestmark = pytest.mark.gpu


def build(rng, t, NL=2, D=256, H=4, KV=2, F=512, V=300, max_seq=64, scaling=None, arch='llama', dense_ends=False,
          v_type=None):
    gen = {8: synth.q8_0, 12: synth.q4_k}[t]
    dev = lambda b: torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()
    hd = D // H
    raw = {'token_embd': synth.q8_0(rng, V, D), 'output': gen(rng, V, D)}
    layers_raw, layers_dev, layers_ref = [], [], []
    for _ in range(NL):
        L = {'attn_q': gen(rng, H * hd, D), 'attn_k': gen(rng, KV * hd, D), 'attn_v': gen(rng, KV * hd, D),
             'attn_output': gen(rng, D, D), 'ffn_gate': gen(rng, F, D), 'ffn_up': gen(rng, F, D),
             'ffn_down': gen(rng, D, F)}
        types = dict.fromkeys(L, t)
        if v_type is not None:                                        # attn_v of another GGML type
            L['attn_v'], types['attn_v'] = synth.make(rng, v_type, KV * hd, D), v_type
        norms = {'attn_norm': (1 + rng.normal(0, 0.1, D)).astype(np.float32),
                 'ffn_norm': (1 + rng.normal(0, 0.1, D)).astype(np.float32)}
        shapes = {'attn_q': (H * hd, D), 'attn_k': (KV * hd, D), 'attn_v': (KV * hd, D), 'attn_output': (D, D),
                  'ffn_gate': (F, D), 'ffn_up': (F, D), 'ffn_down': (D, F)}
        if arch == 'qwen3':                                           # per-head q/k RMSNorm weights
            norms.update({'attn_q_norm': (1 + rng.normal(0, 0.2, hd)).astype(np.float32),
                          'attn_k_norm': (1 + rng.normal(0, 0.2, hd)).astype(np.float32)})
        if arch == 'qwen2':                                           # q/k/v projection biases
            norms.update({'attn_q_bias': rng.normal(0, 0.5, H * hd).astype(np.float32),
                          'attn_k_bias': rng.normal(0, 0.5, KV * hd).astype(np.float32),
                          'attn_v_bias': rng.normal(0, 0.5, KV * hd).astype(np.float32)})
        layers_dev.append({**{k: (dev(v), types[k]) for k, v in L.items()},
                           **{k: torch.from_numpy(v).cuda() for k, v in norms.items()}})
        layers_ref.append({**{k: o.dequantize(v, types[k], shapes[k]).astype(np.float64) for k, v in L.items()},
                           **norms})
    on = (1 + rng.normal(0, 0.1, D)).astype(np.float32)
    weights = {'token_embd': (dev(raw['token_embd']), 8), 'output': (dev(raw['output']), t),
               'output_norm': torch.from_numpy(on).cuda(), 'layers': layers_dev}
    ref_w = {'token_embd': o.dequantize(raw['token_embd'], 8, (V, D)).astype(np.float64),
             'output': o.dequantize(raw['output'], t, (V, D)).astype(np.float64), 'output_norm': on,
             'layers': layers_ref}
    if dense_ends:                         # F16 token embedding, F32 output head (GGML types 1 and 0)
        emb = rng.normal(0, 1, (V, D)).astype(np.float16)
        head = rng.normal(0, D ** -0.5, (V, D)).astype(np.float32)
        weights['token_embd'] = (dev(emb.tobytes()), 1)
        weights['output'] = (dev(head.tobytes()), 0)
        ref_w['token_embd'], ref_w['output'] = emb.astype(np.float64), head.astype(np.float64)
    sc = scaling or {}
    cfg = LlamaConfig(n_layers=NL, d_model=D, n_heads=H, n_kv_heads=KV, d_ff=F, vocab=V, rope_base=10000.0,
                      eps=1e-5, max_seq=max_seq, arch=arch, **sc)
    return QuantLlama(weights, cfg), ref_w, {'n_heads': H, 'n_kv_heads': KV, 'rope_base': 10000.0, 'eps': 1e-5,
                                             'arch': arch, **sc}


@pytest.mark.parametrize('t', [8, 12])
def test_decode_logits_match_oracle(t):
    rng = np.random.default_rng(t)
    model, ref_w, cfg = build(rng, t)
    tokens = [5, 77, 120, 3, 299, 42, 8, 8]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    assert int(model.pos.item()) == len(tokens)
    assert model.tokens[:len(tokens)].cpu().tolist() == [int(np.argmax(r)) for r in ref]


def test_graph_replay_equals_eager_and_greedy_matches_oracle():
    rng = np.random.default_rng(21)
    model, ref_w, cfg = build(rng, 8)
    prompt = [11, 250, 7]
    eager = model.generate(prompt, 6)
    eager_logits = model.logits.clone()
    model.reset()
    model.set_token(prompt[0])
    model.step()                      # eager step before capture
    model.capture()
    got = model.generate(prompt, 6)   # replays the captured step
    torch.cuda.synchronize()
    assert got == eager
    assert torch.equal(model.logits, eager_logits)
    # greedy continuation of the oracle
    seq = list(prompt)
    for _ in range(6):
        seq.append(int(np.argmax(o.llama_decode_f64(ref_w, cfg, seq)[-1])))
    assert got == seq[len(prompt):]


def test_long_context_crosses_attention_chunks():
    """Positions beyond one 128-position attention chunk: logits of the last
    tokens still match the oracle."""
    rng = np.random.default_rng(5)
    model, ref_w, cfg = build(rng, 8, max_seq=320)
    tokens = [int(v) for v in rng.integers(0, 300, size=270)]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        if p in (127, 128, 200, 269):
            torch.cuda.synchronize()
            assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p


@pytest.mark.parametrize('t', [8, 12])
def test_prefill_matches_oracle_then_decode_continues(t):
    """Batched prefill (tensor cores, bf16 weights and activations): last-token
    logits against the float64 oracle, then decoding continues from the cache
    it filled.  Bar 3e-2 normwise: each bf16 tensor-core op stays within 1e-2,
    and two layers of random (untrained) weights compound those roundings."""
    rng = np.random.default_rng(40 + t)
    model, ref_w, cfg = build(rng, t, max_seq=160)
    prompt = [int(v) for v in rng.integers(0, 300, size=70)]       # crosses one 64-position key tile
    ref = o.llama_decode_f64(ref_w, cfg, prompt + [9, 123])
    model.reset()
    model.prefill(prompt)
    torch.cuda.synchronize()
    assert int(model.pos.item()) == len(prompt)
    err = o.normwise_rel_err(model.logits.cpu().numpy(), ref[len(prompt) - 1])
    assert err < 3e-2, ('prefill logits', err)
    for i, tok in enumerate([9, 123]):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        err = o.normwise_rel_err(model.logits.cpu().numpy(), ref[len(prompt) + i])
        assert err < 3e-2, ('decode step after prefill', i, err)


@pytest.mark.parametrize('kind,fac', [('llama3', 8.0), ('linear', 4.0)])
def test_rope_scaling_decode_and_prefill_match_oracle(kind, fac):
    """RoPE scaling (engine/model.py:199-214) through the frequency-table
    kernel: decode logits within 1e-3 of the float64 oracle at every position
    (a short original context puts the 32 frequency pairs in all three llama3
    bands), and the tensor-core prefill within 3e-2.  (These random weights
    make the logits insensitive to RoPE; the kernel's rotation itself is
    checked against the table in test_rope_kv_freq_table.)"""
    rng = np.random.default_rng(61)
    scaling = dict(rope_scaling=kind, rope_factor=fac, rope_orig_ctx=64, rope_low_freq=1.0, rope_high_freq=4.0)
    model, ref_w, cfg = build(rng, 12, max_seq=96, scaling=scaling)
    assert model.inv_freq is not None
    tokens = [int(v) for v in rng.integers(0, 300, size=40)]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    model.reset()
    model.prefill(tokens)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[-1]) < 3e-2


@pytest.mark.parametrize('arch', ['qwen2', 'qwen3'])
def test_qwen_layouts_decode_and_prefill_match_oracle(arch):
    """Qwen2 (q/k/v projection biases) and Qwen3 (per-head q/k RMSNorm), both
    with split-half RoPE pairs (engine/model.py:184-221): decode logits within
    1e-3 of the float64 oracle, prefill within 3e-2, greedy tokens equal."""
    rng = np.random.default_rng(71 if arch == 'qwen2' else 72)
    model, ref_w, cfg = build(rng, 12, max_seq=96, arch=arch)
    assert model.neox
    tokens = [int(v) for v in rng.integers(0, 300, size=24)]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    assert model.tokens[:len(tokens)].cpu().tolist() == [int(np.argmax(r)) for r in ref]
    model.reset()
    model.prefill(tokens)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[-1]) < 3e-2


@pytest.mark.parametrize('D,H,KV,window', [(256, 4, 2, 5), (256, 2, 1, 130), (256, 4, 2, 64)])
def test_sliding_window_decode_and_prefill_match_oracle(D, H, KV, window):
    """Sliding-window attention (engine/model.py:222): decode attends to the
    last ``window`` positions (chunks before the window skipped, the chunk
    holding its start trimmed), prefill masks keys outside each row's window;
    logits within 1e-3 (decode) and 3e-2 (prefill) of the float64 oracle over
    enough tokens for the window to slide across attention chunks."""
    rng = np.random.default_rng(80 + window)
    model, ref_w, cfg = build(rng, 8, D=D, H=H, KV=KV, max_seq=320)
    model.cfg.sliding_window = window
    cfg = dict(cfg, sliding_window=window)
    tokens = [int(v) for v in rng.integers(0, 300, size=150 if window > 100 else 90)]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        if p in (window - 1, window, window + 1, len(tokens) - 1) or p % 29 == 0:
            torch.cuda.synchronize()
            assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    model.reset()
    model.prefill(tokens)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[-1]) < 3e-2


def test_unquantised_embedding_and_output_head():
    """An F16 token embedding and an F32 output head (GGUF files often keep
    those unquantised): the device row lookup and the dense GEMV, decode and
    prefill against the float64 oracle."""
    rng = np.random.default_rng(90)
    model, ref_w, cfg = build(rng, 12, max_seq=64, dense_ends=True)
    tokens = [5, 77, 120, 3, 299, 42, 8, 8]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    model.reset()
    model.prefill(tokens)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[-1]) < 3e-2


@pytest.mark.parametrize('H,KV,hd', [(4, 2, 64), (2, 1, 128)])
def test_qkv_bias_norm_kernel(H, KV, hd):
    """b200q_qkv_bias_norm_dev: bias added to every q/k/v value, then each q
    and k head RMS-normalised with its weights; v heads only biased."""
    from localai_b200 import _lib
    rng = np.random.default_rng(H + hd)
    T, eps = 3, 1e-6
    n = (H + 2 * KV) * hd
    qkv = rng.normal(size=(T, n)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    qn, kn = rng.normal(1, 0.2, hd).astype(np.float32), rng.normal(1, 0.2, hd).astype(np.float32)
    ref = (qkv.astype(np.float64) + bias).reshape(T, H + 2 * KV, hd)
    for hh in range(H + KV):
        g = qn if hh < H else kn
        a = ref[:, hh]
        ref[:, hh] = a / np.sqrt(np.mean(a * a, axis=-1, keepdims=True) + eps) * g
    d = torch.from_numpy(qkv).cuda()
    t = lambda a: torch.from_numpy(a).cuda()
    bd, qd, kd = t(bias), t(qn), t(kn)
    lib = _lib.load()
    _lib.check(lib.b200q_qkv_bias_norm_dev(d.data_ptr(), T, H, KV, hd, bd.data_ptr(), qd.data_ptr(), kd.data_ptr(),
                                           eps, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    np.testing.assert_allclose(d.cpu().numpy(), ref.reshape(T, n), rtol=0, atol=2e-5)


@pytest.mark.parametrize('kind,fac', [('llama3', 8.0), ('linear', 4.0)])
def test_rope_kv_freq_table(kind, fac):
    """b200q_rope_kv_ex_dev: pair j of q and k turns by pos * inv_freq[j]
    (the scaled table of rope_inv_freq), not by base^(-j/half); k and v land
    in the caches."""
    from localai_b200 import _lib, ops
    from localai_b200.decoder import rope_inv_freq
    rng = np.random.default_rng(7)
    H, KV, hd, T, max_seq, p0 = 4, 2, 64, 3, 64, 40
    c = LlamaConfig(n_layers=1, d_model=H * hd, n_heads=H, n_kv_heads=KV, d_ff=64, vocab=8, rope_base=10000.0,
                    rope_scaling=kind, rope_factor=fac, rope_orig_ctx=64)
    inv = rope_inv_freq(c, hd)
    plain = 1.0 / 10000.0 ** (np.arange(hd // 2) / (hd // 2))
    assert np.abs(inv - plain).max() > 1e-2 * plain.max()
    qkv = rng.normal(size=(T, (H + 2 * KV) * hd)).astype(np.float32)
    ref = qkv.astype(np.float64).copy()
    for t in range(T):
        ang = (p0 + t) * inv.astype(np.float64)
        cs, sn = np.cos(ang), np.sin(ang)
        for hh in range(H + KV):
            a = ref[t, hh * hd:(hh + 1) * hd]
            e, od = a[0::2].copy(), a[1::2].copy()
            a[0::2], a[1::2] = e * cs - od * sn, e * sn + od * cs
    kc = torch.zeros((max_seq, KV * hd), device='cuda')
    vc = torch.zeros((max_seq, KV * hd), device='cuda')
    qd = torch.from_numpy(qkv).cuda()
    pos = torch.tensor([p0], dtype=torch.int32, device='cuda')
    invd = torch.from_numpy(inv).cuda()
    lib = _lib.load()
    _lib.check(lib.b200q_rope_kv_ex_dev(qd.data_ptr(), T, H, KV, hd, hd, 10000.0, invd.data_ptr(), 0,
                                        pos.data_ptr(), kc.data_ptr(), vc.data_ptr(), max_seq,
                                        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ops.check_device_error()
    np.testing.assert_allclose(qd.cpu().numpy(), ref, rtol=0, atol=5e-5)
    np.testing.assert_allclose(kc[p0:p0 + T].cpu().numpy(), ref[:, H * hd:(H + KV) * hd], rtol=0, atol=5e-5)
    np.testing.assert_allclose(vc[p0:p0 + T].cpu().numpy(), ref[:, (H + KV) * hd:], rtol=0, atol=0)


@pytest.mark.parametrize('T,rotary', [(1, 64), (5, 32), (3, 0)])
def test_rope_kv_store_partial_rotary(T, rotary):
    """b200q_rope_kv_dev: q and k rotated over the first ``rotary`` dims in
    adjacent pairs (engine/model.py:205-217), rotated k and v stored in the
    caches at positions pos..pos+T-1; dims past ``rotary`` pass unchanged."""
    from localai_b200 import _lib, ops
    rng = np.random.default_rng(T + rotary)
    H, KV, hd, max_seq, base, p0 = 4, 2, 64, 16, 10000.0, 7
    qkv = rng.normal(size=(T, (H + 2 * KV) * hd)).astype(np.float32)
    half = rotary // 2
    ref = qkv.astype(np.float64).copy()
    if half:
        inv = 1.0 / base ** (np.arange(half) / half)
        for t in range(T):
            ang = (p0 + t) * inv
            c, s = np.cos(ang), np.sin(ang)
            for hh in range(H + KV):
                a = ref[t, hh * hd:hh * hd + rotary]
                e, od = a[0::2].copy(), a[1::2].copy()
                a[0::2], a[1::2] = e * c - od * s, e * s + od * c
    kc = torch.full((max_seq, KV * hd), float('nan'), device='cuda')
    vc = torch.full((max_seq, KV * hd), float('nan'), device='cuda')
    qd = torch.from_numpy(qkv).cuda()
    pos = torch.tensor([p0], dtype=torch.int32, device='cuda')
    lib = _lib.load()
    _lib.check(lib.b200q_rope_kv_dev(qd.data_ptr(), T, H, KV, hd, rotary, base, pos.data_ptr(), kc.data_ptr(),
                                     vc.data_ptr(), max_seq, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ops.check_device_error()
    np.testing.assert_allclose(qd.cpu().numpy(), ref, rtol=0, atol=2e-5)
    k_ref = ref[:, H * hd:(H + KV) * hd]
    v_ref = ref[:, (H + KV) * hd:]
    np.testing.assert_allclose(kc[p0:p0 + T].cpu().numpy(), k_ref, rtol=0, atol=2e-5)
    np.testing.assert_allclose(vc[p0:p0 + T].cpu().numpy(), v_ref, rtol=0, atol=0)
    assert torch.isnan(kc[:p0]).all() and torch.isnan(kc[p0 + T:]).all()


def test_rope_kv_position_out_of_range_is_reported():
    from localai_b200 import _lib, ops
    lib = _lib.load()
    qkv = torch.zeros((2, 8 * 64), device='cuda')
    kc = torch.zeros((4, 2 * 64), device='cuda')
    vc = torch.zeros((4, 2 * 64), device='cuda')
    pos = torch.tensor([3], dtype=torch.int32, device='cuda')        # 3 + 2 > max_seq 4
    _lib.check(lib.b200q_rope_kv_dev(qkv.data_ptr(), 2, 4, 2, 64, 64, 10000.0, pos.data_ptr(), kc.data_ptr(),
                                     vc.data_ptr(), 4, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    with pytest.raises(_lib.B200QError):
        ops.check_device_error()
    assert not kc.any() and not vc.any()


def test_head_dim_128_grouped_query_decode_and_prefill():
    """The Llama-3-8B head shape (head dim 128, four query heads per KV head):
    decode steps at 1e-3 and a 70-token prefill (two key tiles) at the bf16
    bar, against the float64 oracle."""
    rng = np.random.default_rng(128)
    model, ref_w, cfg = build(rng, 8, NL=1, D=512, H=4, KV=1, F=256, max_seq=96)
    tokens = [int(v) for v in rng.integers(0, 300, size=6)]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    prompt = [int(v) for v in rng.integers(0, 300, size=70)]
    ref = o.llama_decode_f64(ref_w, cfg, prompt)
    model.reset()
    model.prefill(prompt)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[-1]) < 3e-2


def _write_model_gguf(path, rng, arch, tied, prefix, extra=()):
    """A two-layer Q8_0 model written as a GGUF file under the reference's
    tensor names and metadata keys, and its float64 oracle weights."""
    from localai_b200.gguf import write_gguf
    NL, D, H, KV, F, V = 2, 256, 4, 2, 512, 300
    hd = D // H
    shapes = {'attn_q': (H * hd, D), 'attn_k': (KV * hd, D), 'attn_v': (KV * hd, D), 'attn_output': (D, D),
              'ffn_gate': (F, D), 'ffn_up': (F, D), 'ffn_down': (D, F)}
    f32 = lambda v: (v.astype(np.float32).tobytes(), 0, v.shape)
    tensors, layers = {}, []
    for i in range(NL):
        p, L = f'{prefix}.{i}.', {}
        for k, s in shapes.items():
            raw = synth.q8_0(rng, *s)
            tensors[p + k + '.weight'] = (raw, 8, s)
            L[k] = o.dequantize(raw, 8, s).astype(np.float64)
        for k, name in (('attn_norm', 'attn_norm'), ('ffn_norm', 'post_attention_norm' if arch == 'qwen3'
                                                                  else 'ffn_norm')):
            L[k] = (1 + rng.normal(0, 0.1, D)).astype(np.float32)
            tensors[p + name + '.weight'] = f32(L[k])
        if arch == 'qwen3':                       # per-head q/k norms: 'blk.' names only (engine/model.py:188-192)
            for k in ('attn_q_norm', 'attn_k_norm'):
                L[k] = (1 + rng.normal(0, 0.2, hd)).astype(np.float32)
                tensors[f'blk.{i}.{k}.weight'] = f32(L[k])
        if arch == 'qwen2':                       # q and v biases stored, k's absent (adds nothing)
            for k, n in (('attn_q', H * hd), ('attn_v', KV * hd)):
                L[k + '_bias'] = rng.normal(0, 0.5, n).astype(np.float32)
                tensors[p + k + '.bias'] = f32(L[k + '_bias'])
            L['attn_k_bias'] = np.zeros(KV * hd, np.float32)
        layers.append(L)
    emb = synth.q8_0(rng, V, D)
    on = (1 + rng.normal(0, 0.1, D)).astype(np.float32)
    tensors['token_embd.weight'] = (emb, 8, (V, D))
    tensors['output_norm.weight'] = f32(on)
    ref = {'token_embd': o.dequantize(emb, 8, (V, D)).astype(np.float64), 'output_norm': on, 'layers': layers}
    if tied:
        ref['output'] = ref['token_embd']
    else:
        out = synth.q8_0(rng, V, D)
        tensors['output.weight'] = (out, 8, (V, D))
        ref['output'] = o.dequantize(out, 8, (V, D)).astype(np.float64)
    for name, v in extra:
        tensors[name] = f32(v)
    meta = {'general.architecture': arch, f'{arch}.block_count': NL, f'{arch}.attention.head_count': H,
            f'{arch}.attention.head_count_kv': KV, f'{arch}.embedding_length': D,
            f'{arch}.feed_forward_length': F, f'{arch}.attention.layer_norm_rms_epsilon': 1e-5,
            'tokenizer.ggml.vocab_size': V}
    write_gguf(path, meta, tensors)
    return ref, {'n_heads': H, 'n_kv_heads': KV, 'eps': 1e-5, 'arch': arch}


@pytest.mark.parametrize('arch,tied,prefix', [('llama', False, 'blk'), ('qwen3', True, 'blk'),
                                              ('qwen2', False, 'model.layers')])
def test_from_gguf_matches_oracle(tmp_path, arch, tied, prefix):
    """QuantLlama.from_gguf on a GGUF file with the reference's names and
    metadata (engine/model.py:12-33,174-240): configuration, layer prefixes,
    Qwen3's post-attention norm and q/k norms, Qwen2's biases, tied output
    weights; logits and greedy tokens against the float64 oracle."""
    from localai_b200.gguf import DeviceGGUF
    ref_w, ocfg = _write_model_gguf(tmp_path / 'm.gguf', np.random.default_rng(31), arch, tied, prefix)
    g = DeviceGGUF(tmp_path / 'm.gguf')
    model = QuantLlama.from_gguf(g, max_seq=32)
    c = model.cfg
    assert (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.vocab, c.arch) == (2, 256, 4, 2, 512, 300, arch)
    assert c.rope_base == (10000.0 if arch == 'llama' else 1000000.0)
    ocfg['rope_base'] = c.rope_base
    tokens = [5, 77, 120, 3, 299, 42]
    ref = o.llama_decode_f64(ref_w, ocfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    assert model.tokens[:len(tokens)].cpu().tolist() == [int(np.argmax(r)) for r in ref]


def test_from_gguf_refuses_bias_outside_qkv(tmp_path):
    from localai_b200.gguf import DeviceGGUF
    rng = np.random.default_rng(32)
    _write_model_gguf(tmp_path / 'm.gguf', rng, 'llama', False, 'blk',
                      extra=[('blk.1.ffn_down.bias', rng.normal(size=256))])
    with pytest.raises(ValueError, match='ffn_down.bias'):
        QuantLlama.from_gguf(DeviceGGUF(tmp_path / 'm.gguf'), max_seq=32)


def test_constructor_rejects_short_weights():
    """A matrix shorter than the configured shape is refused on the host,
    before any kernel could read past its end."""
    rng = np.random.default_rng(33)
    model, _, _ = build(rng, 8)
    w = {'token_embd': (model.emb, model.t_emb), 'output': (model.out_w[:-34], model.t_out),
         'output_norm': model.out_norm, 'layers': []}
    with pytest.raises(ValueError, match='output'):
        QuantLlama(w, model.cfg)


@pytest.mark.parametrize('v_type', [14, 8])
def test_mixed_qkv_types_decode_and_prefill(v_type):
    """Q4_K q and k with a Q6_K (or Q8_0) attn_v, as mixed quantisations
    store them: three products into the qkv slices, in the decode step (GEMVs,
    1e-3) and in the prefill (tensor-core GEMMs writing column slices, bf16
    bar), against the float64 oracle."""
    rng = np.random.default_rng(40 + v_type)
    model, ref_w, cfg = build(rng, 12, v_type=v_type)
    assert model.layers[0]['qkv'] is None
    tokens = [5, 77, 120, 3, 299, 42, 8]
    ref = o.llama_decode_f64(ref_w, cfg, tokens)
    model.reset()
    for p, tok in enumerate(tokens):
        model.set_token(tok)
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    prompt = [int(v) for v in rng.integers(0, 300, size=40)]
    ref = o.llama_decode_f64(ref_w, cfg, prompt)
    model.reset()
    model.prefill(prompt)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[-1]) < 3e-2


@pytest.mark.parametrize('variant', ['llama', 'qwen3', 'qwen2'])
def test_from_gguf_matches_the_reference_on_the_same_file(tmp_path, variant):
    """QuantLlama.from_gguf against the reference's own GGUFFile +
    LlamaModel.forward run on the same bytes (tests/golden/llama_gguf_golden.npz,
    files rebuilt from their seed and checked by SHA-256): logits after every
    token within 1e-3, greedy tokens equal."""
    import hashlib
    import importlib.util
    from pathlib import Path
    from localai_b200.gguf import DeviceGGUF
    gold_dir = Path(__file__).resolve().parent / 'golden'
    spec = importlib.util.spec_from_file_location('make_llama_gguf_golden', gold_dir / 'make_llama_gguf_golden.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    gold = np.load(gold_dir / 'llama_gguf_golden.npz')
    path = tmp_path / f'{variant}.gguf'
    mod.build_file(variant, path)
    assert hashlib.sha256(path.read_bytes()).hexdigest() == str(gold[f'{variant}_sha256'])
    model = QuantLlama.from_gguf(DeviceGGUF(path), max_seq=16)
    ref = gold[f'{variant}_logits']
    model.reset()
    for p, tok in enumerate(gold['tokens']):
        model.set_token(int(tok))
        model.step()
        torch.cuda.synchronize()
        assert o.normwise_rel_err(model.logits.cpu().numpy(), ref[p]) < 1e-3, p
    assert model.tokens[:len(ref)].cpu().tolist() == [int(np.argmax(r)) for r in ref]
