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


def build(rng, t, NL=2, D=256, H=4, KV=2, F=512, V=300, max_seq=64):
    gen = {8: synth.q8_0, 12: synth.q4_k}[t]
    dev = lambda b: torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()
    hd = D // H
    raw = {'token_embd': synth.q8_0(rng, V, D), 'output': gen(rng, V, D)}
    layers_raw, layers_dev, layers_ref = [], [], []
    for _ in range(NL):
        L = {'attn_q': gen(rng, H * hd, D), 'attn_k': gen(rng, KV * hd, D), 'attn_v': gen(rng, KV * hd, D),
             'attn_output': gen(rng, D, D), 'ffn_gate': gen(rng, F, D), 'ffn_up': gen(rng, F, D),
             'ffn_down': gen(rng, D, F)}
        norms = {'attn_norm': (1 + rng.normal(0, 0.1, D)).astype(np.float32),
                 'ffn_norm': (1 + rng.normal(0, 0.1, D)).astype(np.float32)}
        shapes = {'attn_q': (H * hd, D), 'attn_k': (KV * hd, D), 'attn_v': (KV * hd, D), 'attn_output': (D, D),
                  'ffn_gate': (F, D), 'ffn_up': (F, D), 'ffn_down': (D, F)}
        layers_dev.append({**{k: (dev(v), t) for k, v in L.items()}, **{k: torch.from_numpy(v).cuda() for k, v in norms.items()}})
        layers_ref.append({**{k: o.dequantize(v, t, shapes[k]).astype(np.float64) for k, v in L.items()}, **norms})
    on = (1 + rng.normal(0, 0.1, D)).astype(np.float32)
    weights = {'token_embd': (dev(raw['token_embd']), 8), 'output': (dev(raw['output']), t),
               'output_norm': torch.from_numpy(on).cuda(), 'layers': layers_dev}
    ref_w = {'token_embd': o.dequantize(raw['token_embd'], 8, (V, D)).astype(np.float64),
             'output': o.dequantize(raw['output'], t, (V, D)).astype(np.float64), 'output_norm': on,
             'layers': layers_ref}
    cfg = LlamaConfig(n_layers=NL, d_model=D, n_heads=H, n_kv_heads=KV, d_ff=F, vocab=V, rope_base=10000.0,
                      eps=1e-5, max_seq=max_seq)
    return QuantLlama(weights, cfg), ref_w, {'n_heads': H, 'n_kv_heads': KV, 'rope_base': 10000.0, 'eps': 1e-5}


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
