"""CPU tests of the decoder configuration read from GGUF metadata, against the
rules of the reference's LlamaModel constructor (engine/model.py:12-33): the
'<arch>.' key first, then 'llama.', then the default; required sizes; the
vocabulary from the tokenizer keys; the RoPE base default by architecture.
Pinned to the reference's own constructor by the committed fixture
tests/golden/llama_config_reference.json."""
import pytest

from localai_b200.decoder import llama_config_from_gguf
from localai_b200.gguf import parse_gguf, write_gguf


def base(arch='llama', **extra):
    m = {'general.architecture': arch, f'{arch}.block_count': 32, f'{arch}.attention.head_count': 32,
         f'{arch}.embedding_length': 4096, f'{arch}.feed_forward_length': 14336,
         'tokenizer.ggml.vocab_size': 128256}
    m.update(extra)
    return m


def test_llama_defaults():
    c = llama_config_from_gguf(base(), max_seq=512)
    assert (c.n_layers, c.d_model, c.n_heads, c.d_ff, c.vocab) == (32, 4096, 32, 14336, 128256)
    assert c.n_kv_heads == 32                      # defaults to the query heads
    assert c.rope_base == 10000.0 and c.rope_dim == 128 and c.eps == 1e-5
    assert (c.rope_scaling, c.rope_factor, c.rope_orig_ctx, c.rope_low_freq, c.rope_high_freq) == \
        ('none', 1.0, 8192, 1.0, 4.0)
    assert c.arch == 'llama' and c.sliding_window == 0 and c.max_seq == 512


def test_llama3_keys():
    c = llama_config_from_gguf(base(**{'llama.attention.head_count_kv': 8, 'llama.rope.freq_base': 500000.0,
                                       'llama.attention.layer_norm_rms_epsilon': 1e-6,
                                       'llama.rope.scaling.type': 'LLAMA3', 'llama.rope.scaling.factor': 8.0,
                                       'llama.rope.scaling.original_context_length': 8192,
                                       'llama.rope.scaling.low_freq_factor': 1.0,
                                       'llama.rope.scaling.high_freq_factor': 4.0,
                                       'llama.rope.dimension_count': 64}))
    assert c.n_kv_heads == 8 and c.rope_base == 500000.0 and c.eps == 1e-6
    assert c.rope_scaling == 'llama3' and c.rope_factor == 8.0 and c.rope_dim == 64


@pytest.mark.parametrize('arch', ['qwen2', 'qwen3'])
def test_qwen_rope_base_default_and_llama_fallback(arch):
    c = llama_config_from_gguf(base(arch))
    assert c.arch == arch and c.rope_base == 1000000.0
    # a key absent under '<arch>.' is read under 'llama.'
    m = base(arch, **{'llama.attention.head_count_kv': 4, f'{arch}.rope.freq_base': 2.0e6})
    c = llama_config_from_gguf(m)
    assert c.n_kv_heads == 4 and c.rope_base == 2.0e6


def test_sliding_window_read_under_the_architecture_only():
    assert llama_config_from_gguf(base('qwen2', **{'llama.attention.sliding_window': 64})).sliding_window == 0
    assert llama_config_from_gguf(base('qwen2', **{'qwen2.attention.sliding_window': 64})).sliding_window == 64


def test_vocab_from_token_list():
    m = base()
    del m['tokenizer.ggml.vocab_size']
    m['tokenizer.ggml.tokens'] = ['a', 'b', 'c']
    assert llama_config_from_gguf(m).vocab == 3


def test_unscaled_types_read_as_none():
    # only llama3 and linear scale RoPE in the reference; another type leaves it unscaled
    c = llama_config_from_gguf(base(**{'llama.rope.scaling.type': 'yarn', 'llama.rope.scaling.factor': 4.0}))
    assert c.rope_scaling == 'none'


@pytest.mark.parametrize('drop', ['llama.block_count', 'llama.attention.head_count', 'llama.embedding_length',
                                  'llama.feed_forward_length', 'tokenizer.ggml.vocab_size'])
def test_missing_required_metadata(drop):
    m = base()
    del m[drop]
    with pytest.raises(ValueError, match='Missing required'):
        llama_config_from_gguf(m)


def test_heads_must_divide_embedding_and_arch_supported():
    with pytest.raises(ValueError, match='divisible'):
        llama_config_from_gguf(base(**{'llama.attention.head_count': 30}))
    with pytest.raises(ValueError, match='unsupported architecture'):
        llama_config_from_gguf(base('gemma2'))


def test_round_trip_through_a_gguf_file(tmp_path):
    """Values as the GGUF encoding stores them (ints, f32 floats, strings)."""
    m = base(**{'llama.attention.head_count_kv': 8, 'llama.rope.freq_base': 500000.0,
                'llama.rope.scaling.type': 'linear', 'llama.rope.scaling.factor': 2.0})
    write_gguf(tmp_path / 'm.gguf', m, {})
    _, meta, _, _ = parse_gguf((tmp_path / 'm.gguf').read_bytes())
    c = llama_config_from_gguf(meta)
    assert (c.n_layers, c.n_kv_heads, c.vocab, c.rope_base, c.rope_scaling, c.rope_factor) == \
        (32, 8, 128256, 500000.0, 'linear', 2.0)


def test_matches_the_reference_constructor():
    """Every case of tests/golden/llama_config_reference.json (made by running
    the reference's own LlamaModel.__init__, make_llama_config_golden.py):
    the same fields, or the same error and message.  The scaling type is
    compared by effect: the reference applies only 'llama3' and 'linear' and
    leaves any other stored type unscaled, which this configuration reads as
    'none'."""
    import json
    from pathlib import Path
    gold = json.loads((Path(__file__).resolve().parent / 'golden' / 'llama_config_reference.json').read_text())
    assert len(gold) >= 13
    names = {'arch': 'arch', 'n_layers': 'n_layers', 'n_heads': 'n_heads', 'n_kv_heads': 'n_kv_heads',
             'dim': 'd_model', 'ffn': 'd_ff', 'vocab': 'vocab', 'eps': 'eps', 'rope_base': 'rope_base',
             'rope_dim': 'rope_dim', 'rope_scaling_factor': 'rope_factor', 'rope_original_context': 'rope_orig_ctx',
             'rope_low_freq': 'rope_low_freq', 'rope_high_freq': 'rope_high_freq', 'sliding_window': 'sliding_window'}
    for case, rec in gold.items():
        if 'error' in rec:
            with pytest.raises(ValueError) as e:
                llama_config_from_gguf(rec['metadata'])
            assert rec['error'] == 'ValueError' and str(e.value) == rec['message'], case
            continue
        c = llama_config_from_gguf(rec['metadata'])
        ref = rec['fields']
        for k, ours in names.items():
            assert getattr(c, ours) == ref[k], (case, k)
        kind = ref['rope_scaling_type'] if ref['rope_scaling_type'] in ('llama3', 'linear') else 'none'
        assert c.rope_scaling == kind, case
