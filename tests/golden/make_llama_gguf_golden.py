"""Generate tests/golden/llama_gguf_golden.npz: the reference's own GGUF
reader and decoder (``GGUFFile`` + ``LlamaModel.forward``, engine/gguf_parser.py
and engine/model.py:12-33,174-240) run token by token on three small GGUF
files, one per tensor layout the decoder resolves by name:

* 'llama': 'blk.<i>.' names, a separate output matrix;
* 'qwen3': 'blk.<i>.' names, Qwen3's 'post_attention_norm' and per-head q/k
  norms, no output matrix (tied to the token embedding);
* 'qwen2': 'model.layers.<i>.' names, q and v projection biases (k's absent),
  'tok_embeddings.weight' and 'norm.weight' instead of 'token_embd' /
  'output_norm'.

Layer matrices are Q8_0, norms and biases F32.  The files are not committed:
``build_file`` writes them from a fixed seed, and the fixture keeps each
file's SHA-256 beside the reference's logits, so a test rebuilds the same
bytes and checks them first.  The reference's native kernels are switched off
for the run, so its products are its exact dequantise-then-f32 path.

    python tests/golden/make_llama_gguf_golden.py <reference checkout>
"""
import hashlib
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

TOKENS = [5, 77, 120, 3, 299, 42]
VARIANTS = ('llama', 'qwen3', 'qwen2')
NL, D, H, KV, F, V = 2, 256, 4, 2, 512, 300


def build_file(variant, path):
    """Write the seeded GGUF file of ``variant`` to ``path``."""
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from localai_b200 import synth
    from localai_b200.gguf import write_gguf
    arch = variant
    rng = np.random.default_rng({'llama': 501, 'qwen3': 502, 'qwen2': 503}[variant])
    hd = D // H
    prefix = 'model.layers' if variant == 'qwen2' else 'blk'
    f32 = lambda a: (np.asarray(a, np.float32).tobytes(), 0, np.asarray(a).shape)
    q8 = lambda r, c: (synth.q8_0(rng, r, c), 8, (r, c))
    t = {}
    for i in range(NL):
        p = f'{prefix}.{i}.'
        for k, (r, c) in (('attn_q', (H * hd, D)), ('attn_k', (KV * hd, D)), ('attn_v', (KV * hd, D)),
                          ('attn_output', (D, D)), ('ffn_gate', (F, D)), ('ffn_up', (F, D)), ('ffn_down', (D, F))):
            t[p + k + '.weight'] = q8(r, c)
        t[p + 'attn_norm.weight'] = f32(1 + rng.normal(0, 0.1, D))
        t[p + ('post_attention_norm' if variant == 'qwen3' else 'ffn_norm') + '.weight'] = f32(1 + rng.normal(0, 0.1, D))
        if variant == 'qwen3':
            for k in ('attn_q_norm', 'attn_k_norm'):
                t[f'blk.{i}.{k}.weight'] = f32(1 + rng.normal(0, 0.2, hd))
        if variant == 'qwen2':
            t[p + 'attn_q.bias'] = f32(rng.normal(0, 0.5, H * hd))
            t[p + 'attn_v.bias'] = f32(rng.normal(0, 0.5, KV * hd))
    emb_name, norm_name = ('tok_embeddings.weight', 'norm.weight') if variant == 'qwen2' else \
        ('token_embd.weight', 'output_norm.weight')
    t[emb_name] = q8(V, D)
    t[norm_name] = f32(1 + rng.normal(0, 0.1, D))
    if variant != 'qwen3':
        t['output.weight'] = q8(V, D)
    meta = {'general.architecture': arch, f'{arch}.block_count': NL, f'{arch}.attention.head_count': H,
            f'{arch}.attention.head_count_kv': KV, f'{arch}.embedding_length': D, f'{arch}.feed_forward_length': F,
            f'{arch}.attention.layer_norm_rms_epsilon': 1e-5, 'tokenizer.ggml.vocab_size': V}
    write_gguf(path, meta, t)


def main(ref_root):
    tmp = Path(tempfile.mkdtemp())
    shutil.copytree(Path(ref_root) / 'engine', tmp / 'engine')
    sys.path.insert(0, str(tmp))
    import engine.native_quant as nq                                 # noqa: E402
    nq._LIB, nq._TRIED = None, True                                  # exact f32 products, no native kernels
    from engine.gguf_parser import GGUFFile                          # noqa: E402
    from engine.model import LlamaModel                              # noqa: E402

    out = {'tokens': np.asarray(TOKENS, np.int32)}
    for variant in VARIANTS:
        path = tmp / f'{variant}.gguf'
        build_file(variant, path)
        with GGUFFile(path) as g:
            m = LlamaModel(g, max_seq=16)
            logits = np.stack([np.asarray(m.forward(tok, pos), np.float32) for pos, tok in enumerate(TOKENS)])
        out[f'{variant}_logits'] = logits
        out[f'{variant}_sha256'] = np.asarray(hashlib.sha256(path.read_bytes()).hexdigest())
        print(variant, logits.shape, [int(np.argmax(r)) for r in logits])
    dst = Path(__file__).resolve().parent / 'llama_gguf_golden.npz'
    np.savez_compressed(dst, **out)
    print(f'wrote {dst}')


if __name__ == '__main__':
    main(sys.argv[1])
