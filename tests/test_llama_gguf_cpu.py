"""CPU checks of the GGUF decoder fixture (tests/golden/llama_gguf_golden.npz,
made by running the reference's GGUFFile + LlamaModel.forward on three
seeded files): the files rebuild byte for byte, and the float64 decoder
oracle, given the tensors read from each file by the reference's names,
reproduces the reference's logits."""
import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest

from oracle import quant_oracle as o
from localai_b200.gguf import parse_gguf

GOLD = Path(__file__).resolve().parent / 'golden'


def fixture_module():
    spec = importlib.util.spec_from_file_location('make_llama_gguf_golden', GOLD / 'make_llama_gguf_golden.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def oracle_weights(buf, variant, mod):
    """The oracle's weight dict from the file, by the names the reference
    resolves (engine/model.py:174-240)."""
    _, meta, tensors, _ = parse_gguf(buf)

    def val(name):
        x = tensors[name]
        raw = buf[x.offset:x.offset + x.nbytes]
        if x.ggml_type == 0:
            return np.frombuffer(raw, np.float32).reshape(x.shape).astype(np.float64)
        return o.dequantize(raw, x.ggml_type, x.shape).astype(np.float64)

    prefix = 'model.layers' if variant == 'qwen2' else 'blk'
    layers = []
    for i in range(mod.NL):
        p = f'{prefix}.{i}.'
        L = {k: val(p + k + '.weight') for k in ('attn_q', 'attn_k', 'attn_v', 'attn_output', 'ffn_gate', 'ffn_up',
                                                 'ffn_down', 'attn_norm')}
        L['ffn_norm'] = val(p + ('post_attention_norm' if variant == 'qwen3' else 'ffn_norm') + '.weight')
        for k in ('attn_q_norm', 'attn_k_norm'):
            if f'blk.{i}.{k}.weight' in tensors:
                L[k] = val(f'blk.{i}.{k}.weight')
        if any(p + k + '.bias' in tensors for k in ('attn_q', 'attn_k', 'attn_v')):
            for k, n in (('attn_q', mod.H * mod.D // mod.H), ('attn_k', mod.KV * mod.D // mod.H),
                         ('attn_v', mod.KV * mod.D // mod.H)):
                L[k + '_bias'] = val(p + k + '.bias') if p + k + '.bias' in tensors else np.zeros(n)
        layers.append(L)
    emb = 'tok_embeddings.weight' if 'tok_embeddings.weight' in tensors else 'token_embd.weight'
    norm = 'norm.weight' if 'norm.weight' in tensors else 'output_norm.weight'
    w = {'token_embd': val(emb), 'output_norm': val(norm), 'layers': layers}
    w['output'] = val('output.weight') if 'output.weight' in tensors else w['token_embd']
    cfg = {'n_heads': mod.H, 'n_kv_heads': mod.KV, 'eps': float(np.float32(1e-5)), 'arch': variant,
           'rope_base': 10000.0 if variant == 'llama' else 1000000.0}
    return w, cfg


@pytest.mark.parametrize('variant', ['llama', 'qwen3', 'qwen2'])
def test_fixture_files_rebuild_and_oracle_matches_reference(tmp_path, variant):
    mod = fixture_module()
    gold = np.load(GOLD / 'llama_gguf_golden.npz')
    path = tmp_path / f'{variant}.gguf'
    mod.build_file(variant, path)
    buf = path.read_bytes()
    assert hashlib.sha256(buf).hexdigest() == str(gold[f'{variant}_sha256'])
    w, cfg = oracle_weights(buf, variant, mod)
    ref = o.llama_decode_f64(w, cfg, [int(t) for t in gold['tokens']])
    got = gold[f'{variant}_logits']
    for p in range(len(gold['tokens'])):
        assert o.normwise_rel_err(got[p], ref[p]) < 1e-5, p
