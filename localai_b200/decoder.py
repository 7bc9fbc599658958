"""Greedy decode of the reference's Llama decoder on the GPU.

``engine/model.py:174-240`` (``LlamaModel.forward``, arch 'llama' / 'qwen2' /
'qwen3', RoPE plain or scaled: llama3 / linear) runs one token through every
layer with NumPy and the native quantised matvecs.  ``QuantLlama`` keeps
every weight on the device in its raw
GGUF form and runs one token per *step*:

    x = emb[token]                                  b200q_dequant_row_dev
    per layer:
        h = rmsnorm(x) * attn_norm                  b200q_add_rmsnorm_dev
        qkv = [Wq; Wk; Wv] h                        b200q_gemv_dev (one GEMV)
        rope(q, k); cache[pos] = k, v               b200q_rope_kv_dev
        att = softmax(q k^T / sqrt(hd)) v           b200q_attn_decode_ex_dev
        x += Wo att; h = rmsnorm(x) * ffn_norm      b200q_gemv_dev, b200q_add_rmsnorm_dev
        x += Wdown silu([Wgate; Wup] h)             b200q_gemv_dev, b200q_silu_mul_dev, b200q_gemv_dev
    logits = Wout (rmsnorm(x) * output_norm)        b200q_gemv_dev
    token = argmax(logits); pos += 1                b200q_argmax_dev

The position and the token live in device memory, so a step is captured once
in a CUDA graph and replayed per token without host synchronisation
(``capture()``); prompt tokens are fed by overwriting the device token before
each step.

``prefill(tokens)`` runs a whole prompt at once (``LlamaModel.forward_sequence``,
engine/model.py:118-170): embedding rows, then per layer RMSNorm (bf16 out),
the tensor-core GEMMs (QKV, O, gate/up with fused SiLU*up, down) over all
prompt rows, RoPE and the KV-cache store for every row, and causal
grouped-query attention (on the tensor cores, ``b200q_attn_prefill_tc_dev``,
for head dim 128; else the f32 ``b200q_attn_prefill_dev``); the last row goes
through the output head and argmax like a decode step, so decoding continues
from there.  bf16 tensor-core operands: logits within 1e-2 of the f32 path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, ops
from .moe import _stream


@dataclass
class LlamaConfig:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_ff: int
    vocab: int
    rope_base: float = 10000.0
    rope_dim: int | None = None       # default: head_dim
    eps: float = 1e-5
    max_seq: int = 2048
    # RoPE scaling, as the GGUF keys {arch}.rope.scaling.* (engine/model.py:
    # 21-26): 'none', 'llama3' (Llama 3.1/3.2 frequency interpolation) or
    # 'linear' (angles divided by the factor); only applied for factor > 1
    rope_scaling: str = 'none'
    rope_factor: float = 1.0
    rope_orig_ctx: int = 8192
    rope_low_freq: float = 1.0
    rope_high_freq: float = 4.0
    # 'llama' (adjacent RoPE pairs) or 'qwen2' / 'qwen3' (split-half NeoX pairs,
    # engine/model.py:212-221); Qwen2 layers may carry q/k/v biases and Qwen3
    # layers per-head q/k norms (the optional 'attn_{q,k,v}_bias' and
    # 'attn_{q,k}_norm' entries of a layer's weights)
    arch: str = 'llama'
    # {arch}.attention.sliding_window: a query attends to the last this many
    # positions (engine/model.py:222); 0 = all
    sliding_window: int = 0

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


DECODER_ARCHS = ('llama', 'qwen2', 'qwen3')


def llama_config_from_gguf(metadata: dict, max_seq: int = 2048) -> LlamaConfig:
    """The decoder configuration from GGUF metadata, read the way
    engine/model.py:12-33 reads it: '<arch>.<key>' first, then
    'llama.<key>', then the reference's default (KV heads = heads; RMS eps
    1e-5; RoPE base 1e6 for qwen2/qwen3, else 1e4; RoPE dims = head dim;
    scaling 'none', factor 1, original context 8192, low/high frequency
    factors 1 and 4; sliding window 0, read from '<arch>.' only); the
    vocabulary from tokenizer.ggml.vocab_size or the length of the token list.
    Raises ValueError, as the reference does, when a required size is missing
    or the heads do not divide the embedding, and for architectures other than
    llama / qwen2 / qwen3."""
    m = metadata

    def meta(*keys, default=None):
        for k in keys:
            if k in m:
                return m[k]
        return default

    arch = str(meta('general.architecture', default='llama'))
    if arch not in DECODER_ARCHS:
        raise ValueError(f'unsupported architecture {arch!r} (supported: {", ".join(DECODER_ARCHS)})')

    def key(name, default=None):
        return meta(f'{arch}.{name}', f'llama.{name}', default=default)

    n_layers = int(key('block_count', 0))
    n_heads = int(key('attention.head_count', 0))
    n_kv = int(key('attention.head_count_kv', n_heads))
    dim = int(key('embedding_length', 0))
    ffn = int(key('feed_forward_length', 0))
    vocab = int(meta('tokenizer.ggml.vocab_size', default=len(m.get('tokenizer.ggml.tokens', []))))
    if not all((n_layers, n_heads, n_kv, dim, ffn, vocab)):
        raise ValueError(f'Missing required Llama architecture metadata for {arch!r}')
    if dim % n_heads:
        raise ValueError('embedding_length must be divisible by attention.head_count')
    # the reference applies only these two scalings (engine/model.py:199-214);
    # any other stored type leaves RoPE unscaled there, and so here
    scaling = str(key('rope.scaling.type', 'none')).lower()
    if scaling not in ('llama3', 'linear'):
        scaling = 'none'
    return LlamaConfig(
        n_layers=n_layers, d_model=dim, n_heads=n_heads, n_kv_heads=n_kv, d_ff=ffn, vocab=vocab,
        rope_base=float(key('rope.freq_base', 1000000.0 if arch in ('qwen2', 'qwen3') else 10000.0)),
        rope_dim=int(key('rope.dimension_count', dim // n_heads)),
        eps=float(key('attention.layer_norm_rms_epsilon', 1e-5)), max_seq=max_seq,
        rope_scaling=scaling,
        rope_factor=float(key('rope.scaling.factor', 1.0)),
        rope_orig_ctx=int(key('rope.scaling.original_context_length', 8192)),
        rope_low_freq=float(key('rope.scaling.low_freq_factor', 1.0)),
        rope_high_freq=float(key('rope.scaling.high_freq_factor', 4.0)),
        arch=arch, sliding_window=int(meta(f'{arch}.attention.sliding_window', default=0) or 0))


def rope_inv_freq(cfg: LlamaConfig, rotary: int):
    """Per-pair RoPE frequencies with the configured scaling, or None for
    plain base^(-j / half).  float32 arithmetic in the order of the reference
    (engine/model.py:199-214): llama3 keeps the high-frequency pairs, divides
    the low-frequency ones by the factor and blends the band between; linear
    divides every angle by the factor (folded into the frequency here)."""
    import numpy as np
    kind = cfg.rope_scaling.lower()
    if kind not in ('none', 'llama3', 'linear'):
        raise ValueError(f'unsupported RoPE scaling {cfg.rope_scaling!r}')
    half = rotary // 2
    if kind == 'none' or cfg.rope_factor <= 1.0 or half == 0:
        return None
    f32 = np.float32
    inv = (f32(1.0) / (f32(cfg.rope_base) ** (np.arange(half, dtype=f32) / f32(max(half, 1))))).astype(f32)
    fac = f32(cfg.rope_factor)
    if kind == 'linear':
        return (inv / fac).astype(f32)
    orig, lo, hi = f32(cfg.rope_orig_ctx), f32(cfg.rope_low_freq), f32(cfg.rope_high_freq)
    wavelength = (f32(2.0 * np.pi) / np.maximum(inv, f32(1e-12))).astype(f32)
    low_wl = orig / max(lo, f32(1e-6))
    high_wl = orig / max(hi, f32(1e-6))
    smooth = ((orig / np.maximum(wavelength, f32(1e-12)) - lo) / max(hi - lo, f32(1e-6))).astype(f32)
    blended = ((f32(1.0) - smooth) * (inv / fac) + smooth * inv).astype(f32)
    return np.where(wavelength > low_wl, inv / fac, np.where(wavelength < high_wl, inv, blended)).astype(f32)


class QuantLlama:
    """``weights``: ``{'token_embd': (raw, type), 'output': (raw, type),
    'output_norm': f32, 'layers': [ {'attn_q': (raw, type), 'attn_k', 'attn_v',
    'attn_output', 'ffn_gate', 'ffn_up', 'ffn_down': (raw, type),
    'attn_norm': f32, 'ffn_norm': f32}, ... ]}`` with raw uint8 CUDA tensors of
    GGUF blocks (rows = output features) and f32 CUDA norm vectors."""

    def __init__(self, weights: dict, cfg: LlamaConfig):
        self.cfg = c = cfg
        if c.d_model % c.n_heads or c.n_heads % c.n_kv_heads:
            raise ValueError('heads must divide d_model and kv heads must divide heads')
        self.lib = _lib.load()
        hd = c.head_dim
        self.rotary = min(c.rope_dim or hd, hd)
        self.rotary -= self.rotary % 2
        dev = weights['output_norm'].device
        self.dev = dev
        inv = rope_inv_freq(c, self.rotary)
        self.inv_freq = None if inv is None else torch.from_numpy(inv).to(dev)
        if c.sliding_window < 0:
            raise ValueError('sliding_window must be >= 0')
        if c.arch not in ('llama', 'qwen2', 'qwen3'):
            raise ValueError(f'unsupported architecture {c.arch!r}')
        self.neox = c.arch != 'llama'
        D, F, qd, kvd = c.d_model, c.d_ff, c.n_heads * hd, c.n_kv_heads * hd

        # every matrix and vector is checked against the configured shape before
        # any kernel reads it (a short buffer would otherwise be read past its end)
        def check_mat(name, w, rows, cols):
            try:
                ops._check_weights(w[0], w[1], rows, cols)
            except ValueError as e:
                raise ValueError(f'{name}: {e} ({rows} x {cols} expected)') from None

        def check_vec(name, v, n):
            if v is not None and (not v.is_cuda or v.numel() != n):
                raise ValueError(f'{name}: expected a CUDA vector of {n} values')

        check_mat('token_embd', weights['token_embd'], c.vocab, D)
        check_mat('output', weights['output'], c.vocab, D)
        check_vec('output_norm', weights['output_norm'], D)
        if len(weights['layers']) != c.n_layers:
            raise ValueError(f'{len(weights["layers"])} layers of weights for n_layers={c.n_layers}')
        for i, lw in enumerate(weights['layers']):
            for name, rows, cols in (('attn_q', qd, D), ('attn_k', kvd, D), ('attn_v', kvd, D), ('attn_output', D, qd),
                                     ('ffn_gate', F, D), ('ffn_up', F, D), ('ffn_down', D, F)):
                check_mat(f'layer {i} {name}', lw[name], rows, cols)
            for name, n in (('attn_norm', D), ('ffn_norm', D), ('attn_q_bias', qd), ('attn_k_bias', kvd),
                            ('attn_v_bias', kvd), ('attn_q_norm', hd), ('attn_k_norm', hd)):
                check_vec(f'layer {i} {name}', lw.get(name), n)
            if any(k in lw for k in ('attn_q_bias', 'attn_k_bias', 'attn_v_bias')):
                missing = [k for k in ('attn_q_bias', 'attn_k_bias', 'attn_v_bias') if k not in lw]
                if missing:
                    raise ValueError(f'layer {i}: q/k/v biases come together (missing {", ".join(missing)})')
        self.emb, self.t_emb = weights['token_embd']
        self.out_w, self.t_out = weights['output']
        self.out_norm = weights['output_norm'].float().contiguous()
        self.layers = []
        for lw in weights['layers']:
            tq, tk, tv = lw['attn_q'][1], lw['attn_k'][1], lw['attn_v'][1]
            if lw['ffn_up'][1] != lw['ffn_gate'][1]:
                raise ValueError('ffn_gate and ffn_up must share their GGML type')
            same = tq == tk == tv
            self.layers.append({
                # q, k and v of one GGML type: one product over the stacked rows;
                # of different types (a Q6_K attn_v beside Q4_K q and k, as mixed
                # quantisations store them): three products into the slices of qkv
                'qkv': (torch.cat([lw['attn_q'][0].reshape(-1), lw['attn_k'][0].reshape(-1),
                                   lw['attn_v'][0].reshape(-1)]), tq) if same else None,
                'qkv_parts': None if same else [(lw['attn_q'][0], tq, 0, qd), (lw['attn_k'][0], tk, qd, kvd),
                                                (lw['attn_v'][0], tv, qd + kvd, kvd)],
                'o': lw['attn_output'],
                'gu': (torch.cat([lw['ffn_gate'][0].reshape(-1), lw['ffn_up'][0].reshape(-1)]), lw['ffn_gate'][1]),
                'down': lw['ffn_down'],
                'attn_norm': lw['attn_norm'].float().contiguous(),
                'ffn_norm': lw['ffn_norm'].float().contiguous(),
                'qkv_bias': (torch.cat([lw['attn_q_bias'], lw['attn_k_bias'], lw['attn_v_bias']]).float().contiguous()
                             if 'attn_q_bias' in lw else None),
                'q_norm': lw['attn_q_norm'].float().contiguous() if 'attn_q_norm' in lw else None,
                'k_norm': lw['attn_k_norm'].float().contiguous() if 'attn_k_norm' in lw else None,
            })
        f32 = dict(dtype=torch.float32, device=dev)
        kvd = c.n_kv_heads * hd
        self.k_cache = torch.zeros((c.n_layers, c.max_seq, kvd), **f32)
        self.v_cache = torch.zeros((c.n_layers, c.max_seq, kvd), **f32)
        self.x = torch.zeros(c.d_model, **f32)
        self.h = torch.zeros(c.d_model, **f32)
        self.qkv = torch.zeros(c.n_heads * hd + 2 * kvd, **f32)
        self.att = torch.zeros(c.d_model, **f32)
        self.o = torch.zeros(c.d_model, **f32)
        self.gu = torch.zeros(2 * c.d_ff, **f32)
        self.act = torch.zeros(c.d_ff, **f32)
        self.dn = torch.zeros(c.d_model, **f32)
        self.logits = torch.zeros(c.vocab, **f32)
        self.scratch = torch.zeros(self.lib.b200q_attn_decode_scratch_floats(c.n_heads, hd, c.max_seq), **f32)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(c.max_seq, dtype=torch.int32, device=dev)   # argmax after position p
        self.amax_key = torch.zeros(1, dtype=torch.int64, device=dev)         # grid-wide argmax word
        self.emb_row_bytes = ops.row_bytes(self.t_emb, c.d_model)
        self.graph = None

    @classmethod
    def from_gguf(cls, gguf, max_seq: int = 2048) -> 'QuantLlama':
        """A decoder over the tensors of a ``DeviceGGUF`` (already on the
        device, blocks kept raw), configured by ``llama_config_from_gguf`` and
        found by the names engine/model.py:174-240 looks up: per layer
        'blk.<i>.' or 'model.layers.<i>.' + attn_norm, attn_q, attn_k, attn_v,
        attn_output, ffn_norm ('post_attention_norm' for qwen3), ffn_gate,
        ffn_up, ffn_down ('.weight'); the optional per-head 'blk.<i>.attn_q_norm'
        / 'attn_k_norm' and q/k/v '.bias' tensors (a missing one of the three
        biases reads as zeros); 'token_embd' (or 'tok_embeddings'),
        'output_norm' (or 'norm') and 'output', the token embedding standing in
        for a missing output matrix (tied weights), as the reference does.  The
        vocabulary is the output matrix's row count (the length of the
        reference's logits).  A bias stored for any other matrix raises
        ValueError: this decoder adds biases to q, k and v only."""
        from dataclasses import replace
        cfg = llama_config_from_gguf(gguf.metadata, max_seq)
        tensors = gguf.tensors

        def layer_name(i, suffix):
            for n in (f'blk.{i}.{suffix}', f'model.layers.{i}.{suffix}'):
                if n in tensors:
                    return n
            raise KeyError(f'Missing tensor for layer {i}: {suffix}')

        def mat(name, biased=False):
            x = tensors[name]
            if len(x.shape) != 2:
                raise ValueError(f'{name}: expected a matrix, got shape {x.shape}')
            if not biased and name.endswith('.weight') and name[:-6] + 'bias' in tensors:
                raise ValueError(f'{name[:-6]}bias: biases are supported on attn_q / attn_k / attn_v only')
            return gguf.raw(name), x.ggml_type

        def vec(name):
            return gguf.tensor_dev(name).reshape(-1).float().contiguous()

        emb = gguf.find('token_embd.weight', 'tok_embeddings.weight')
        out_norm = gguf.find('output_norm.weight', 'norm.weight')
        if emb is None or out_norm is None:
            raise KeyError('missing token_embd.weight or output_norm.weight')
        out = gguf.find('output.weight') or emb
        cfg = replace(cfg, vocab=int(tensors[out].shape[0]))
        hd = cfg.head_dim
        ffn_norm = 'post_attention_norm.weight' if cfg.arch == 'qwen3' else 'ffn_norm.weight'
        layers = []
        for i in range(cfg.n_layers):
            lw = {k: mat(layer_name(i, k + '.weight')) for k in ('attn_output', 'ffn_gate', 'ffn_up', 'ffn_down')}
            lw['attn_norm'] = vec(layer_name(i, 'attn_norm.weight'))
            lw['ffn_norm'] = vec(layer_name(i, ffn_norm))
            qkv = {k: layer_name(i, k + '.weight') for k in ('attn_q', 'attn_k', 'attn_v')}
            biased = any(n[:-6] + 'bias' in tensors for n in qkv.values())
            for k, rows in (('attn_q', cfg.n_heads * hd), ('attn_k', cfg.n_kv_heads * hd),
                            ('attn_v', cfg.n_kv_heads * hd)):
                lw[k] = mat(qkv[k], biased=True)
                b = qkv[k][:-6] + 'bias'
                if biased:
                    lw[k + '_bias'] = (vec(b) if b in tensors
                                       else torch.zeros(rows, dtype=torch.float32, device=gguf.device))
            for k in ('attn_q_norm', 'attn_k_norm'):
                if f'blk.{i}.{k}.weight' in tensors:
                    lw[k] = vec(f'blk.{i}.{k}.weight')
            layers.append(lw)
        # the embedding is read by rows, and as a tied output matrix without a
        # bias (engine/model.py:176-180,236-240): no bias check for it
        weights = {'token_embd': mat(emb, biased=True), 'output': mat(out, biased=out == emb),
                   'output_norm': vec(out_norm), 'layers': layers}
        return cls(weights, cfg)

    # -- one step -------------------------------------------------------------
    def _rope(self, qkv, T, kc, vc, st, L=None):
        """Optional q/k/v bias and per-head q/k norms (layer L), then RoPE of T
        rows of qkv at positions pos.. and their k/v cache store (a frequency
        table when RoPE scaling is configured; split-half pairs for Qwen)."""
        c, lib, hd = self.cfg, self.lib, self.cfg.head_dim
        if L is not None and (L['qkv_bias'] is not None or L['q_norm'] is not None or L['k_norm'] is not None):
            ptr = lambda t: None if t is None else t.data_ptr()
            _lib.check(lib.b200q_qkv_bias_norm_dev(qkv.data_ptr(), T, c.n_heads, c.n_kv_heads, hd, ptr(L['qkv_bias']),
                                                   ptr(L['q_norm']), ptr(L['k_norm']), c.eps, st))
        if self.inv_freq is None and not self.neox:
            _lib.check(lib.b200q_rope_kv_dev(qkv.data_ptr(), T, c.n_heads, c.n_kv_heads, hd, self.rotary, c.rope_base,
                                             self.pos.data_ptr(), kc.data_ptr(), vc.data_ptr(), c.max_seq, st))
        else:
            _lib.check(lib.b200q_rope_kv_ex_dev(qkv.data_ptr(), T, c.n_heads, c.n_kv_heads, hd, self.rotary, c.rope_base,
                                                None if self.inv_freq is None else self.inv_freq.data_ptr(),
                                                1 if self.neox else 0, self.pos.data_ptr(), kc.data_ptr(),
                                                vc.data_ptr(), c.max_seq, st))

    def _gemv(self, w, x, y, rows, cols):
        raw, t = w
        _lib.check(self.lib.b200q_gemv_dev(t, raw.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, 1, rows, 1,
                                           _stream()))

    def _qkv_gemv(self, L):
        if L['qkv'] is not None:
            self._gemv(L['qkv'], self.h, self.qkv, self.qkv.numel(), self.cfg.d_model)
        else:
            for raw, t, o0, n in L['qkv_parts']:
                self._gemv((raw, t), self.h, self.qkv[o0:o0 + n], n, self.cfg.d_model)

    def _step(self):
        c, lib, st = self.cfg, self.lib, _stream()
        hd = c.head_dim
        _lib.check(lib.b200q_dequant_row_dev(self.t_emb, self.emb.data_ptr(), self.emb_row_bytes, c.d_model,
                                             self.token.data_ptr(), c.vocab, 1, self.x.data_ptr(), st))
        delta = None
        for li, L in enumerate(self.layers):
            _lib.check(lib.b200q_add_rmsnorm_dev(self.x.data_ptr(), None if delta is None else delta.data_ptr(),
                                                 L['attn_norm'].data_ptr(), 1, c.d_model, c.eps, self.h.data_ptr(),
                                                 None, st))
            self._qkv_gemv(L)
            kc, vc = self.k_cache[li], self.v_cache[li]
            self._rope(self.qkv, 1, kc, vc, st, L)
            _lib.check(lib.b200q_attn_decode_ex_dev(self.qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                    self.pos.data_ptr(), c.n_heads, c.n_kv_heads, hd, c.max_seq,
                                                    c.sliding_window, self.scratch.data_ptr(), self.att.data_ptr(),
                                                    st))
            self._gemv(L['o'], self.att, self.o, c.d_model, c.d_model)
            _lib.check(lib.b200q_add_rmsnorm_dev(self.x.data_ptr(), self.o.data_ptr(), L['ffn_norm'].data_ptr(), 1,
                                                 c.d_model, c.eps, self.h.data_ptr(), None, st))
            self._gemv(L['gu'], self.h, self.gu, 2 * c.d_ff, c.d_model)
            _lib.check(lib.b200q_silu_mul_dev(self.gu.data_ptr(), 1, c.d_ff, self.act.data_ptr(), c.d_ff, st))
            self._gemv(L['down'], self.act, self.dn, c.d_model, c.d_ff)
            delta = self.dn
        _lib.check(lib.b200q_add_rmsnorm_dev(self.x.data_ptr(), delta.data_ptr(), self.out_norm.data_ptr(), 1,
                                             c.d_model, c.eps, self.h.data_ptr(), None, st))
        self._gemv((self.out_w, self.t_out), self.h, self.logits, c.vocab, c.d_model)
        _lib.check(lib.b200q_argmax_dev(self.logits.data_ptr(), c.vocab, self.token.data_ptr(), self.pos.data_ptr(),
                                        self.tokens.data_ptr(), c.max_seq, self.amax_key.data_ptr(), st))

    # -- batched prompt --------------------------------------------------------
    def _gemm_w(self, key, w, rows, cols):
        """16-byte-row copy of a weight for the tensor-core path (made once)."""
        cache = self.__dict__.setdefault('_gemm_cache', {})
        if key not in cache:
            raw, t = w
            cache[key] = ops.pad_rows(raw, rows, ops.packed_row_bytes(t, cols)) + (t,)
        return cache[key]

    def prefill(self, tokens: list[int]) -> None:
        """All prompt tokens at positions pos, pos+1, ... in one pass; leaves
        the argmax of the last token in ``tokens[pos + len - 1]`` and advances
        pos by len(tokens)."""
        c, lib, st = self.cfg, self.lib, _stream()
        T = len(tokens)
        if T < 1:
            raise ValueError('empty prompt')
        dev, hd = self.dev, c.head_dim
        kvd = c.n_kv_heads * hd
        nq = c.n_heads * hd + 2 * kvd
        ids = torch.tensor(tokens, dtype=torch.int32, device=dev)
        X = torch.empty((T, c.d_model), dtype=torch.float32, device=dev)
        _lib.check(lib.b200q_dequant_row_dev(self.t_emb, self.emb.data_ptr(), self.emb_row_bytes, c.d_model,
                                             ids.data_ptr(), c.vocab, T, X.data_ptr(), st))
        Hb = torch.empty((T, c.d_model), dtype=torch.bfloat16, device=dev)
        qkv = torch.empty((T, nq), dtype=torch.float32, device=dev)
        attb = torch.empty((T, c.d_model), dtype=torch.bfloat16, device=dev)
        O = torch.empty((T, c.d_model), dtype=torch.float32, device=dev)
        act = torch.empty((T, c.d_ff), dtype=torch.bfloat16, device=dev)
        Dn = torch.empty((T, c.d_model), dtype=torch.float32, device=dev)
        off = torch.tensor([0, T], dtype=torch.int32, device=dev)
        # head dim 128: causal attention on the tensor cores (bf16 staging copies in
        # scratch); a sliding window takes the f32 kernel, which masks it
        scratch = None
        if hd == 128 and c.sliding_window <= 0:
            nb = lib.b200q_attn_prefill_tc_scratch_bytes(T, c.n_heads, c.n_kv_heads, hd, c.max_seq)
            scratch = torch.empty(nb, dtype=torch.uint8, device=dev)
        delta = None
        for li, L in enumerate(self.layers):
            _lib.check(lib.b200q_add_rmsnorm_dev(X.data_ptr(), None if delta is None else delta.data_ptr(),
                                                 L['attn_norm'].data_ptr(), T, c.d_model, c.eps, None, Hb.data_ptr(),
                                                 st))
            if L['qkv'] is not None:
                wq, sq, tq = self._gemm_w(('qkv', li), L['qkv'], nq, c.d_model)
                ops.gemm_quant(Hb, wq, off, k=c.d_model, n_feat=nq, w_rows_per_group=nq, ggml_type=tq,
                               w_row_bytes=sq, out=qkv)
            else:                      # column slices of qkv (row stride nq)
                for j, (raw, t, o0, n) in enumerate(L['qkv_parts']):
                    wj, sj, tj = self._gemm_w(('qkv', li, j), (raw, t), n, c.d_model)
                    ops.gemm_quant(Hb, wj, off, k=c.d_model, n_feat=n, w_rows_per_group=n, ggml_type=tj,
                                   w_row_bytes=sj, out=qkv[:, o0:o0 + n])
            kc, vc = self.k_cache[li], self.v_cache[li]
            self._rope(qkv, T, kc, vc, st, L)
            if scratch is not None:
                _lib.check(lib.b200q_attn_prefill_tc_dev(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                         self.pos.data_ptr(), T, c.n_heads, c.n_kv_heads, hd,
                                                         c.max_seq, scratch.data_ptr(), scratch.numel(),
                                                         attb.data_ptr(), st))
            else:
                _lib.check(lib.b200q_attn_prefill_ex_dev(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                         self.pos.data_ptr(), T, c.n_heads, c.n_kv_heads, hd,
                                                         c.max_seq, c.sliding_window, attb.data_ptr(), st))
            wo, so, to = self._gemm_w(('o', li), L['o'], c.d_model, c.d_model)
            ops.gemm_quant(attb, wo, off, k=c.d_model, n_feat=c.d_model, w_rows_per_group=c.d_model, ggml_type=to,
                           w_row_bytes=so, out=O)
            _lib.check(lib.b200q_add_rmsnorm_dev(X.data_ptr(), O.data_ptr(), L['ffn_norm'].data_ptr(), T, c.d_model,
                                                 c.eps, None, Hb.data_ptr(), st))
            wg, sg, tg = self._gemm_w(('gu', li), L['gu'], 2 * c.d_ff, c.d_model)
            ops.gemm_quant(Hb, wg, off, k=c.d_model, n_feat=c.d_ff, w_rows_per_group=2 * c.d_ff, up_offset=c.d_ff,
                           ggml_type=tg, w_row_bytes=sg, act=act)
            wd, sd, td = self._gemm_w(('down', li), L['down'], c.d_model, c.d_ff)
            ops.gemm_quant(act, wd, off, k=c.d_ff, n_feat=c.d_model, w_rows_per_group=c.d_model, ggml_type=td,
                           w_row_bytes=sd, out=Dn)
            delta = Dn
        # last row -> output head, as a decode step
        self.x.copy_(X[T - 1])
        _lib.check(lib.b200q_add_rmsnorm_dev(self.x.data_ptr(), Dn[T - 1].data_ptr(), self.out_norm.data_ptr(), 1,
                                             c.d_model, c.eps, self.h.data_ptr(), None, st))
        self._gemv((self.out_w, self.t_out), self.h, self.logits, c.vocab, c.d_model)
        self.pos.add_(T - 1)
        _lib.check(lib.b200q_argmax_dev(self.logits.data_ptr(), c.vocab, self.token.data_ptr(), self.pos.data_ptr(),
                                        self.tokens.data_ptr(), c.max_seq, self.amax_key.data_ptr(), st))

    def step(self):
        """One token through the model (graph replay once captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step()

    def capture(self):
        """Capture one step in a CUDA graph (after one eager step has set up
        every kernel's attributes).  Replays reuse the same buffers."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = g

    # -- driving ------------------------------------------------------------
    def reset(self):
        self.pos.zero_()
        self.token.zero_()

    def set_token(self, token: int):
        self.token.fill_(int(token))

    def generate(self, prompt: list[int], n_new: int) -> list[int]:
        """Greedy continuation of ``prompt`` (reference: repetition penalty 1,
        argmax sampling).  Returns the n_new generated token ids."""
        c = self.cfg
        if not prompt or len(prompt) + n_new > c.max_seq:
            raise ValueError('prompt + new tokens must fit max_seq')
        self.reset()
        for t in prompt:
            self.set_token(t)
            self.step()
        for _ in range(n_new - 1):
            self.step()
        p = len(prompt)
        return self.tokens[p - 1:p - 1 + n_new].tolist()

    def logits_at(self) -> torch.Tensor:
        """Logits of the last step."""
        return self.logits
