"""CPU tests of the GGUF loaders' host logic: which tensors
``QuantLlama.from_gguf`` hands to the decoder for each layout the reference
resolves by name (engine/model.py:174-240), and the shape checks of
``ZayaMoE.from_gguf``.  The files are the seeded ones of
tests/golden/make_llama_gguf_golden.py; a DeviceGGUF stand-in keeps their
tensors in host memory, and the decoder's constructor is replaced by one that
records what it receives (the kernels are tested on the GPU)."""
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from localai_b200.decoder import QuantLlama
from localai_b200.gguf import DeviceGGUF, parse_gguf, write_gguf

GOLD = Path(__file__).resolve().parent / 'golden'


class HostGGUF(DeviceGGUF):
    """DeviceGGUF over host memory (parsing and lookup only)."""

    def __init__(self, path):
        self.buf = Path(path).read_bytes()
        self.version, self.metadata, self.tensors, self.alignment = parse_gguf(self.buf)
        self.device = torch.device('cpu')
        self.device_tensors = {n: torch.frombuffer(bytearray(self.buf[x.offset:x.offset + x.nbytes]),
                                                   dtype=torch.uint8) for n, x in self.tensors.items()}

    def tensor_dev(self, name):
        x = self.tensors[name]
        assert x.ggml_type == 0
        return self.device_tensors[name].view(torch.float32).reshape(x.shape)


def fixture_module():
    spec = importlib.util.spec_from_file_location('make_llama_gguf_golden', GOLD / 'make_llama_gguf_golden.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture
def captured(monkeypatch):
    got = {}

    def record(self, weights, cfg):
        got['weights'], got['cfg'] = weights, cfg
    monkeypatch.setattr(QuantLlama, '__init__', record)
    return got


@pytest.mark.parametrize('variant', ['llama', 'qwen3', 'qwen2'])
def test_decoder_tensors_by_the_reference_names(tmp_path, captured, variant):
    mod = fixture_module()
    path = tmp_path / 'm.gguf'
    mod.build_file(variant, path)
    g = HostGGUF(path)
    QuantLlama.from_gguf(g, max_seq=16)
    w, c = captured['weights'], captured['cfg']
    assert (c.arch, c.n_layers, c.vocab, c.max_seq) == (variant, mod.NL, mod.V, 16)
    prefix = 'model.layers' if variant == 'qwen2' else 'blk'

    def same(t, name):
        return bytes(t.numpy()) == bytes(g.device_tensors[name].numpy())

    for i, L in enumerate(w['layers']):
        p = f'{prefix}.{i}.'
        for k in ('attn_q', 'attn_k', 'attn_v', 'attn_output', 'ffn_gate', 'ffn_up', 'ffn_down'):
            assert same(L[k][0], p + k + '.weight') and L[k][1] == 8, (i, k)
        assert same(L['ffn_norm'].view(torch.uint8),
                    p + ('post_attention_norm' if variant == 'qwen3' else 'ffn_norm') + '.weight')
        assert ('attn_q_norm' in L) == (variant == 'qwen3')
        if variant == 'qwen2':          # q and v biases stored, k's absent: zeros
            assert same(L['attn_q_bias'].view(torch.uint8), p + 'attn_q.bias')
            assert same(L['attn_v_bias'].view(torch.uint8), p + 'attn_v.bias')
            assert not L['attn_k_bias'].any() and L['attn_k_bias'].numel() == mod.KV * mod.D // mod.H
        else:
            assert 'attn_q_bias' not in L
    emb = 'tok_embeddings.weight' if variant == 'qwen2' else 'token_embd.weight'
    assert same(w['token_embd'][0], emb)
    # qwen3 has no output matrix: the token embedding stands in (tied weights)
    assert same(w['output'][0], emb if variant == 'qwen3' else 'output.weight')


def test_decoder_refuses_a_bias_outside_qkv(tmp_path, captured):
    mod = fixture_module()
    path = tmp_path / 'm.gguf'
    mod.build_file('llama', path)
    _, meta, tensors, _ = parse_gguf(path.read_bytes())
    buf = path.read_bytes()
    t = {n: (buf[x.offset:x.offset + x.nbytes], x.ggml_type, x.shape) for n, x in tensors.items()}
    t['output.bias'] = (np.zeros(mod.V, np.float32).tobytes(), 0, (mod.V,))
    write_gguf(tmp_path / 'b.gguf', meta, t)
    with pytest.raises(ValueError, match='output.bias'):
        QuantLlama.from_gguf(HostGGUF(tmp_path / 'b.gguf'))


def test_decoder_missing_layer_tensor(tmp_path, captured):
    mod = fixture_module()
    path = tmp_path / 'm.gguf'
    mod.build_file('llama', path)
    buf = path.read_bytes()
    _, meta, tensors, _ = parse_gguf(buf)
    t = {n: (buf[x.offset:x.offset + x.nbytes], x.ggml_type, x.shape) for n, x in tensors.items()
         if n != 'blk.1.ffn_up.weight'}
    write_gguf(tmp_path / 'c.gguf', meta, t)
    with pytest.raises(KeyError, match='Missing tensor for layer 1: ffn_up.weight'):
        QuantLlama.from_gguf(HostGGUF(tmp_path / 'c.gguf'))


def test_zaya_expert_shapes_checked_before_any_upload(tmp_path):
    from localai_b200 import synth
    from localai_b200.zaya import ZayaMoE
    rng = np.random.default_rng(0)
    E, D, F = 4, 256, 256
    gu = b''.join(synth.q4_k(rng, 2 * F, D) for _ in range(E))
    dn = b''.join(synth.q4_k(rng, D, F) for _ in range(E - 1))       # one expert short
    write_gguf(tmp_path / 'z.gguf', {'general.architecture': 'zaya'},
               {'blk.1.ffn_gate_up_exps.weight': (gu, 12, (E, 2 * F, D)),
                'blk.1.ffn_down_exps.weight': (dn, 12, (E - 1, D, F))})
    with pytest.raises(ValueError, match='does not match'):
        ZayaMoE.from_gguf(HostGGUF(tmp_path / 'z.gguf'), 1)


def test_gguf_product_argument_errors_match_the_reference(tmp_path):
    """matvec / matmul refuse wrong shapes with the reference's messages
    (engine/gguf_parser.py:187-197,297-307), before any device work."""
    mod = fixture_module()
    path = tmp_path / 'm.gguf'
    mod.build_file('llama', path)
    g = HostGGUF(path)
    name, cols = 'blk.0.ffn_gate.weight', mod.D
    v = np.zeros(cols, np.float32)
    cases = [
        (lambda: g.matvec(name, v.reshape(1, -1)), f'{name}: expected vector shape ({cols},), got (1, {cols})'),
        (lambda: g.matvec(name, v[:-1]), f'{name}: expected vector shape ({cols},), got ({cols - 1},)'),
        (lambda: g.matmul(name, v), f'{name}: expected batch shape (tokens, {cols}), got ({cols},)'),
        (lambda: g.matvec(name, v, row_chunk=0), 'row_chunk must be positive'),
        (lambda: g.matmul(name, v.reshape(1, -1), row_chunk=-1), 'row_chunk must be positive'),
        (lambda: g.matvec('blk.0.attn_norm.weight', v),
         f"blk.0.attn_norm.weight: matvec requires a 2-D tensor, got ({cols},)"),
    ]
    for call, msg in cases:
        with pytest.raises(ValueError) as e:
            call()
        assert str(e.value) == msg
