"""Generate tests/golden/llama_config_reference.json by running the reference's
own ``LlamaModel.__init__`` (engine/model.py:12-33) on GGUF metadata alone:
for each metadata dict below, the architecture fields it derives, or the
error it raises.

The stub GGUF carries only ``metadata`` (all the constructor reads); the KV
cache is sized with a tiny ``max_seq``.

    python tests/golden/make_llama_config_golden.py <reference checkout>
"""
import json
import shutil
import sys
import tempfile
from pathlib import Path

FIELDS = ('arch', 'n_layers', 'n_heads', 'n_kv_heads', 'dim', 'ffn', 'vocab', 'eps', 'rope_base', 'rope_dim',
          'rope_scaling_type', 'rope_scaling_factor', 'rope_original_context', 'rope_low_freq', 'rope_high_freq',
          'sliding_window')


def cases():
    def base(arch='llama', **extra):
        m = {'general.architecture': arch, f'{arch}.block_count': 4, f'{arch}.attention.head_count': 8,
             f'{arch}.embedding_length': 512, f'{arch}.feed_forward_length': 1536, 'tokenizer.ggml.vocab_size': 1000}
        m.update(extra)
        return m

    out = {
        'llama_defaults': base(),
        'llama3_scaled': base(**{'llama.attention.head_count_kv': 2, 'llama.rope.freq_base': 500000.0,
                                 'llama.attention.layer_norm_rms_epsilon': 1e-6, 'llama.rope.scaling.type': 'llama3',
                                 'llama.rope.scaling.factor': 8.0,
                                 'llama.rope.scaling.original_context_length': 8192,
                                 'llama.rope.scaling.low_freq_factor': 1.0,
                                 'llama.rope.scaling.high_freq_factor': 4.0, 'llama.rope.dimension_count': 32}),
        'linear_upper_case': base(**{'llama.rope.scaling.type': 'LINEAR', 'llama.rope.scaling.factor': 2.0}),
        'yarn_type_stored': base(**{'llama.rope.scaling.type': 'yarn', 'llama.rope.scaling.factor': 4.0}),
        'qwen2_defaults': base('qwen2', **{'qwen2.attention.head_count_kv': 2}),
        'qwen3_llama_fallback': base('qwen3', **{'llama.attention.head_count_kv': 4, 'qwen3.rope.freq_base': 2.0e6,
                                                 'llama.attention.layer_norm_rms_epsilon': 1e-6}),
        'qwen2_window': base('qwen2', **{'qwen2.attention.sliding_window': 64}),
        'window_under_llama_key_only': base('qwen2', **{'llama.attention.sliding_window': 64}),
        'no_architecture_key': {k: v for k, v in base().items() if k != 'general.architecture'},
        'vocab_from_tokens': {**{k: v for k, v in base().items() if k != 'tokenizer.ggml.vocab_size'},
                              'tokenizer.ggml.tokens': ['a', 'b', 'c', 'd']},
        'missing_block_count': {k: v for k, v in base().items() if k != 'llama.block_count'},
        'missing_vocab': {k: v for k, v in base().items() if k != 'tokenizer.ggml.vocab_size'},
        'heads_do_not_divide': base(**{'llama.attention.head_count': 7}),
    }
    return out


def main(ref_root):
    tmp = Path(tempfile.mkdtemp())
    shutil.copytree(Path(ref_root) / 'engine', tmp / 'engine')
    sys.path.insert(0, str(tmp))
    from engine.model import LlamaModel                              # noqa: E402

    class Stub:
        def __init__(self, metadata):
            self.metadata = metadata

    result = {}
    for name, meta in cases().items():
        try:
            m = LlamaModel(Stub(meta), max_seq=2)
            result[name] = {'metadata': meta, 'fields': {f: getattr(m, f) for f in FIELDS}}
        except Exception as e:                                         # the reference's own refusal
            result[name] = {'metadata': meta, 'error': type(e).__name__, 'message': str(e)}
    out = Path(__file__).resolve().parent / 'llama_config_reference.json'
    out.write_text(json.dumps(result, indent=1, sort_keys=True) + '\n')
    print(f'wrote {out} ({len(result)} cases)')


if __name__ == '__main__':
    main(sys.argv[1])
