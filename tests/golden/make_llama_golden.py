"""Generate tests/golden/llama_decode_golden.npz by running the reference's own
``LlamaModel.forward`` (engine/model.py:174-240) token by token on a tiny
stub model with f32 weights, plain RoPE and with llama3 / linear RoPE scaling,
and in the Qwen2 / Qwen3 layouts.

The stub supplies what ``forward`` touches: ``gguf`` (``metadata``,
``tensors``, ``find``), ``w`` and ``mat`` (a plain f32 ``x @ W.T``, standing in
for the quantised matvecs, which are pinned separately), the KV cache and the
architecture fields of ``LlamaModel.__init__``.

    python tests/golden/make_llama_golden.py <reference checkout>
"""
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np


def main(ref_root):
    tmp = Path(tempfile.mkdtemp())
    shutil.copytree(Path(ref_root) / 'engine', tmp / 'engine')
    sys.path.insert(0, str(tmp))
    from engine.model import LlamaModel, KVCache                     # noqa: E402

    rng = np.random.default_rng(77)
    NL, D, H, KV, F, V = 2, 64, 4, 2, 96, 50
    hd = D // H
    f = lambda *s, sc=1.0: rng.normal(0, sc, size=s).astype(np.float32)
    T = {'token_embd.weight': f(V, D), 'output.weight': f(V, D, sc=D ** -0.5),
         'output_norm.weight': (1 + f(D, sc=0.1)).astype(np.float32)}
    for l in range(NL):
        p = f'blk.{l}.'
        T.update({p + 'attn_q.weight': f(H * hd, D, sc=D ** -0.5), p + 'attn_k.weight': f(KV * hd, D, sc=D ** -0.5),
                  p + 'attn_v.weight': f(KV * hd, D, sc=D ** -0.5), p + 'attn_output.weight': f(D, D, sc=D ** -0.5),
                  p + 'ffn_gate.weight': f(F, D, sc=D ** -0.5), p + 'ffn_up.weight': f(F, D, sc=D ** -0.5),
                  p + 'ffn_down.weight': f(D, F, sc=F ** -0.5), p + 'attn_norm.weight': (1 + f(D, sc=0.1)),
                  p + 'ffn_norm.weight': (1 + f(D, sc=0.1))})

    class GG:
        metadata = {}
        tensors = dict.fromkeys(T)

        def find(self, *names):
            for n in names:
                if n in T:
                    return n
            return None

    m = LlamaModel.__new__(LlamaModel)
    m.gguf = GG()
    m.arch, m.n_layers, m.n_heads, m.n_kv_heads, m.dim, m.ffn, m.vocab = 'llama', NL, H, KV, D, F, V
    m.eps, m.rope_base, m.rope_dim, m.head_dim = 1e-5, 10000.0, hd, hd
    m.rope_scaling_type, m.rope_scaling_factor = 'none', 1.0
    m.rope_original_context, m.rope_low_freq, m.rope_high_freq = 8192, 1.0, 4.0
    m.sliding_window = 0
    m.cache = KVCache(NL, KV, hd, 32)
    m._weights = {}
    m.w = lambda name: T[name]
    m.mat = lambda x, name: (np.asarray(x, np.float32) @ T[name].T).astype(np.float32)
    tokens = [3, 17, 42, 5, 0, 49, 8]
    logits = np.stack([m.forward(t, p) for p, t in enumerate(tokens)]).astype(np.float32)
    # RoPE scaling (engine/model.py:199-214): llama3 interpolation with a short
    # original context, so that the 8 frequency pairs fall in all three bands
    # (kept, blended, divided), and linear; same weights and tokens
    scaled = {}
    for kind, fac in (('llama3', 8.0), ('linear', 4.0)):
        m.rope_scaling_type, m.rope_scaling_factor = kind, fac
        m.rope_original_context, m.rope_low_freq, m.rope_high_freq = 64, 1.0, 4.0
        m.cache = KVCache(NL, KV, hd, 32)
        scaled['logits_' + kind] = np.stack([m.forward(t, p) for p, t in enumerate(tokens)]).astype(np.float32)
    # Qwen layouts (engine/model.py:184-221): split-half RoPE pairs; qwen3 with
    # per-head q/k RMSNorm weights and its FFN norm named post_attention_norm,
    # qwen2 with q/k/v projection biases (added by the reference's own
    # _mat_impl, which these runs use instead of the plain stub matvec)
    extra = {}
    for l in range(NL):
        p = f'blk.{l}.'
        extra[p + 'attn_q_norm.weight'] = (1 + f(hd, sc=0.2)).astype(np.float32)
        extra[p + 'attn_k_norm.weight'] = (1 + f(hd, sc=0.2)).astype(np.float32)
        extra[p + 'post_attention_norm.weight'] = T[p + 'ffn_norm.weight']
        extra[p + 'attn_q.bias'] = f(H * hd, sc=0.5)
        extra[p + 'attn_k.bias'] = f(KV * hd, sc=0.5)
        extra[p + 'attn_v.bias'] = f(KV * hd, sc=0.5)
    m.rope_scaling_type, m.rope_scaling_factor = 'none', 1.0
    for arch in ('qwen3', 'qwen2'):
        keep = (lambda n: 'bias' not in n) if arch == 'qwen3' else (lambda n: 'norm' not in n or 'attn_norm' in n)
        TT = dict(T, **{k: v for k, v in extra.items() if keep(k) and not (arch == 'qwen2' and 'post_attention' in k)})

        class GQ(GG):
            tensors = dict.fromkeys(TT)

            def find(self, *names):
                for n in names:
                    if n in TT:
                        return n
                return None

        m.gguf = GQ()
        m.arch = arch
        m.cache = KVCache(NL, KV, hd, 32)
        m.w = lambda name, TT=TT: TT[name]
        m.mat = lambda x, name: LlamaModel._mat_impl(m, np.asarray(x, np.float32), name).astype(np.float32)
        scaled['logits_' + arch] = np.stack([m.forward(t, p) for p, t in enumerate(tokens)]).astype(np.float32)
    # sliding window of 3 positions (engine/model.py:222), llama layout
    m.gguf, m.arch, m.w = GG(), 'llama', (lambda name: T[name])
    m.mat = lambda x, name: (np.asarray(x, np.float32) @ T[name].T).astype(np.float32)
    m.sliding_window = 3
    m.cache = KVCache(NL, KV, hd, 32)
    scaled['logits_window3'] = np.stack([m.forward(t, p) for p, t in enumerate(tokens)]).astype(np.float32)
    m.sliding_window = 0
    out = Path(__file__).resolve().parent / 'llama_decode_golden.npz'
    np.savez_compressed(out, logits=logits, tokens=np.array(tokens), **scaled,
                        **{k.replace('.', '_'): v for k, v in T.items()},
                        **{k.replace('.', '_'): v for k, v in extra.items()})
    print('wrote', out)


if __name__ == '__main__':
    if len(sys.argv) != 2:
        sys.exit('usage: make_llama_golden.py <reference checkout>')
    main(sys.argv[1])
