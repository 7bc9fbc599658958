"""Benchmark: expert-parallel MoE layer tokens/s (+ quantised GEMV HBM GB/s).

Workload (the headline configuration): one MoE FFN layer with hidden 4096,
64 experts of intermediate 1408 (down weights padded to 1536), top-8 routing
with renormalised weights, Q4_K expert weights, 16384 tokens of f32 N(0,1)
hidden states, and a router bias log(p_e), p_e ~ (e+1)^-1.1 (Zipf s = 1.1).
All inputs are seeded synthetic data; the token count is fixed across GPU
counts (strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs one process per GPU (torchrun); experts are placed by greedy LPT on
the routing loads and exchanged with NCCL all-to-all.  ``--impl reference``
times the reference engine's own CPU kernels (the reference's native_quant.cpp,
compiled from its sources into oracle/_ref/) on a bounded token sample.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

E, D, F, K_TOP, T_TOTAL = 64, 4096, 1408, 8, 16384
T_HEADLINE = T_TOTAL          # the configured token count (--tokens may change T_TOTAL)
F_PAD = 1536
Q4K_BLOCK = 144
WORKLOAD = 'moe_q4k_d4096_e64_f1408_top8_t16384_zipf1.1'
METRIC = 'MoE-layer tokens/s (expert-parallel, 1/2/4/8 GPU); quant GEMV HBM GB/s'
PROFILE_TRAFFIC = ROOT / 'profiles' / 'gemm_q4k_gate_up_moe_config5.txt'


# ----------------------------------------------------------------- workload
def zipf_bias():
    p = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    return np.log(p / p.sum()).astype(np.float32)


def router_weights():
    return np.random.default_rng(1000).normal(0, 1 / np.sqrt(D), size=(E, D)).astype(np.float32)


def expert_weights(e):
    from localai_b200 import synth
    rng = np.random.default_rng(2000 + e)
    return synth.q4_k(rng, 2 * F, D), synth.q4_k(rng, D, F_PAD, zero_tail_cols=F_PAD - F)


def set_tokens(n):
    global T_TOTAL, WORKLOAD
    T_TOTAL = n
    WORKLOAD = f'moe_q4k_d4096_e64_f1408_top8_t{n}_zipf1.1'


def hidden_states(torch, device, t0, t1, seed=1001):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h = torch.randn((T_TOTAL, D), generator=g, device=device, dtype=torch.float32)
    return h[t0:t1].contiguous()


def algorithmic_flops(slots):
    return 2.0 * slots * (2 * F * D + D * F)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index):
        self.gpu_index = str(gpu_index)
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.QUERY}', '--format=csv,noheader,nounits',
                                          '-lms', '200'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0=None, t1=None):
        """Stop sampling; summarise the samples taken in [t0, t1] (the timed
        region).  If the region was shorter than the sampling period, the
        samples of the whole loaded period (warm-up + timed) are used and the
        summary says so."""
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        window = 'timed region'
        lines = [l for (t, l) in self.lines if t0 is None or (t0 <= t <= t1 + 0.2)]
        if not lines:
            window = 'warm-up and timed region (timed region shorter than the 200 ms sampling period)'
            lines = [l for (_, l) in self.lines]
        sm, mx, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in lines:
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9 or f[0] != self.gpu_index:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == 'active':
                    reasons.add(n)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': max(mx), 'reasons': sorted(reasons),
                'samples': len(sm), 'window': window}


# ----------------------------------------------------------------- CPU (reference kernels)
def cpu_reference_moe(tokens, threads=8):
    """Time the reference engine's CPU path on ``tokens`` tokens.

    Router + softmax/top-8 in NumPy, then per expert the reference's own
    batched Q4_K kernel (localai_q4k_matmul, engine/native_quant.cpp:754-758,
    built from the reference sources into oracle/_ref/) for gate/up and
    down, SiLU in NumPy (engine/zaya.py:304-306), weighted combine.  Falls back
    to the NumPy oracle port when the compiled reference is unavailable.
    Returns (tokens/s, kind, cores).
    """
    from oracle import quant_oracle as o
    so = ROOT / 'oracle' / '_ref' / 'libnative_quant_ref.so'
    lib = ctypes.CDLL(str(so)) if so.exists() else None
    cores = min(threads, os.cpu_count() or 1)
    wr = router_weights()
    bias = zipf_bias()
    h = np.random.default_rng(1002).normal(size=(tokens, D)).astype(np.float32)
    ids, w = o.route_topk(h @ wr.T + bias, K_TOP)          # the routing of the sample (untimed below)
    experts = {int(e): expert_weights(int(e)) for e in np.unique(ids)}

    def matmul(raw, x, rows, cols):
        if lib is None:
            return (o.dequantize(raw, 12, (rows, cols)) @ x.T.astype(np.float32)).astype(np.float32)
        out = np.empty((rows, x.shape[0]), np.float32)
        xb = np.ascontiguousarray(x, np.float32)
        rb = np.frombuffer(raw, np.uint8)
        lib.localai_q4k_matmul(rb.ctypes.data_as(ctypes.c_void_p), xb.ctypes.data_as(ctypes.c_void_p),
                               out.ctypes.data_as(ctypes.c_void_p), rows, cols, x.shape[0], cores)
        return out

    t0 = time.perf_counter()
    logits = h @ wr.T + bias
    ids, w = o.route_topk(logits, K_TOP)
    y = np.zeros((tokens, D), np.float32)
    for e in np.unique(ids):
        rows, slots = np.nonzero(ids == e)
        gu_raw, dn_raw = experts[int(e)]
        gu = matmul(gu_raw, h[rows], 2 * F, D)               # [2F, n]
        gate, up = gu[:F], gu[F:]
        act = np.zeros((rows.size, F_PAD), np.float32)
        act[:, :F] = (gate / (1.0 + np.exp(-np.clip(gate, -80, 80))) * up).T
        out = matmul(dn_raw, act, D, F_PAD)                  # [D, n]
        y[rows] += (out * w[rows, slots][None, :]).T
    dt = time.perf_counter() - t0
    return tokens / dt, ('reference' if lib is not None else 'port'), cores, dt


def cpu_reference_extras(threads=8):
    """The reference's CPU path for configurations 1-3 (its own kernels built
    from its sources into oracle/_ref/, ``threads`` pool threads; NumPy SiLU,
    router and top-k as engine/model.py:161-166 and engine/zaya.py:274-307).
    Bounded samples; returns {} when the compiled reference is unavailable."""
    so = ROOT / 'oracle' / '_ref' / 'libnative_quant_ref.so'
    if not so.exists():
        return {}
    from localai_b200 import synth
    from oracle import quant_oracle as o
    lib = ctypes.CDLL(str(so))
    cores = min(threads, os.cpu_count() or 1)
    vp = ctypes.c_void_p

    def mv(fn, raw, x, rows, cols):
        out = np.empty(rows, np.float32)
        xb = np.ascontiguousarray(x, np.float32)
        getattr(lib, fn)(np.frombuffer(raw, np.uint8).ctypes.data_as(vp), xb.ctypes.data_as(vp),
                         out.ctypes.data_as(vp), rows, cols, cores)
        return out

    def mm(fn, raw, x, rows, cols):
        out = np.empty((rows, x.shape[0]), np.float32)
        xb = np.ascontiguousarray(x, np.float32)
        getattr(lib, fn)(np.frombuffer(raw, np.uint8).ctypes.data_as(vp), xb.ctypes.data_as(vp),
                         out.ctypes.data_as(vp), rows, cols, x.shape[0], cores)
        return out

    def timed(f, min_s=0.3, max_reps=200):
        f()
        n, t0 = 0, time.perf_counter()
        while n < max_reps and (n == 0 or time.perf_counter() - t0 < min_s):
            f()
            n += 1
        return (time.perf_counter() - t0) / n

    silu = lambda g: g / (1.0 + np.exp(-np.clip(g, -80, 80)))
    res = {'cores': cores, 'kind': 'reference'}
    rng = np.random.default_rng(5)
    # configuration 1: Q4_K GEMV 4096 x 4096
    w1 = synth.q4_k(rng, 4096, 4096)
    x1 = rng.normal(size=4096).astype(np.float32)
    t1 = timed(lambda: mv('localai_q4k_matvec', w1, x1, 4096, 4096))
    res['config1_gemv'] = {'us_per_call': round(t1 * 1e6, 1), 'GB_s': round(9469952 / t1 / 1e9, 2)}
    # configuration 2: dense Q4_K FFN (gate/up 14336 x 4096, down 4096 x 14336)
    g2, u2, d2 = synth.q4_k(rng, 14336, 4096), synth.q4_k(rng, 14336, 4096), synth.q4_k(rng, 4096, 14336)

    def ffn1():
        x = x1
        return mv('localai_q4k_matvec', d2, silu(mv('localai_q4k_matvec', g2, x, 14336, 4096)) *
                  mv('localai_q4k_matvec', u2, x, 14336, 4096), 4096, 14336)
    t2 = timed(ffn1)
    X = rng.normal(size=(512, 4096)).astype(np.float32)

    def ffn512():
        gt = mm('localai_q4k_matmul', g2, X, 14336, 4096)
        ut = mm('localai_q4k_matmul', u2, X, 14336, 4096)
        return mm('localai_q4k_matmul', d2, (silu(gt) * ut).T, 4096, 14336)
    t512 = timed(ffn512, min_s=0.0, max_reps=1)
    res['config2_dense_ffn'] = {'T1_us': round(t2 * 1e6, 1), 'T512_ms': round(t512 * 1e3, 1),
                                'T512_TFLOP_s': round(180388626432.0 / t512 / 1e12, 4)}
    # configuration 3: Q6_K MoE (D 2048, 16 experts, F 1024, top-2), ZAYA-style per-token matvecs
    E3, D3, F3 = 16, 2048, 1024
    gu3 = [synth.q6_k(rng, 2 * F3, D3) for _ in range(E3)]
    dn3 = [synth.q6_k(rng, D3, F3) for _ in range(E3)]
    wr3 = rng.normal(0, 0.02, size=(E3, D3)).astype(np.float32)
    H = rng.normal(size=(64, D3)).astype(np.float32)

    def moe_tokens(n):
        ids, w = o.route_topk(H[:n] @ wr3.T, 2)
        for t in range(n):
            for j in range(2):
                e = int(ids[t, j])
                gu = mv('localai_q6k_matvec', gu3[e], H[t], 2 * F3, D3)
                mv('localai_q6k_matvec', dn3[e], silu(gu[:F3]) * gu[F3:], D3, F3) * w[t, j]
    t_1 = timed(lambda: moe_tokens(1))
    t_64 = timed(lambda: moe_tokens(64), min_s=0.0, max_reps=1)
    res['config3_moe_q6k'] = {'T1_us': round(t_1 * 1e6, 1), 'T64_tokens_per_s': round(64 / t_64, 1),
                              'path': 'per-token router + native Q6_K matvecs (engine/zaya.py:274-307)'}
    # configuration 4: one Q8_0 decode token = 32 layers x (q, k, v, o, gate, up, down) + output matvec;
    # one layer's matvecs and a 1/8 slice of the output matrix are timed and extrapolated
    Dm, Ff, KVd = 4096, 14336, 1024
    mats = [(synth.q8_0(rng, r, c_), r, c_) for r, c_ in ((Dm, Dm), (KVd, Dm), (KVd, Dm), (Dm, Dm), (Ff, Dm), (Ff, Dm),
                                                          (Dm, Ff))]
    outs = synth.q8_0(rng, 128256 // 8, Dm)
    xs = {Dm: rng.normal(size=Dm).astype(np.float32), Ff: rng.normal(size=Ff).astype(np.float32)}
    t_layer = timed(lambda: [mv('localai_q8_0_matvec', m, xs[c_], r, c_) for m, r, c_ in mats], min_s=0.5, max_reps=5)
    t_outs = timed(lambda: mv('localai_q8_0_matvec', outs, xs[Dm], 128256 // 8, Dm), min_s=0.2, max_reps=10)
    t_tok = 32 * t_layer + 8 * t_outs
    res['config4_decode_q8_0'] = {'decode_tokens_per_s': round(1.0 / t_tok, 3), 'ms_per_token': round(t_tok * 1e3, 1),
                                  'sample': 'one layer of matvecs x 32 + 1/8 of the output matrix x 8 '
                                            '(matvecs only; attention and norms not included)'}
    return res


def run_reference_arm(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    tokens = args.cpu_tokens
    vals = []
    for i in range(args.warmup + args.steps):
        v, kind, cores, dt = cpu_reference_moe(tokens)
        if i >= args.warmup:
            vals.append(v)
    value = float(np.mean(vals))
    line = {'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': 'tokens/s', 'n_gpus': args.gpus,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': tokens / value * 1e3,
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic',
            'config': {'workload': WORKLOAD, 'sample_tokens': tokens},
            'cpu_baseline': {'value': value, 'unit': 'tokens/s', 'cores': cores, 'kind': kind,
                             'sample': f'{tokens} of {T_TOTAL} tokens per step, all experts they route to'},
            'e2e': {'value': value, 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU arm
def gemv_probe(torch, ops, synth, hbm_peak):
    """Config-1 Q4_K GEMV (4096 x 4096, batch 1) and a 14336 x 4096 one, in a
    CUDA graph over weight copies that together exceed twice the L2."""
    res = {}
    for rows, cols in ((4096, 4096), (14336, 4096)):
        raw = synth.q4_k(np.random.default_rng(1), rows, cols)
        w0 = torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()
        ncopy = max(2, int(300e6 // len(raw)) + 1)
        ws = [w0.clone() for _ in range(ncopy)]
        x = torch.randn(1, cols, device='cuda')
        y = torch.empty(1, rows, device='cuda')
        reps = 60
        for i in range(3):
            ops.gemv(ws[i % ncopy], x, 12, rows, cols, out=y)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(reps):
                    ops.gemv(ws[i % ncopy], x, 12, rows, cols, out=y)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (5 * reps)
        nbytes = len(raw) + 4 * cols + 4 * rows
        gbs = nbytes / (us * 1e-6) / 1e9
        res[f'{rows}x{cols}'] = {'us_per_call': round(us, 2), 'GB_s': round(gbs, 1),
                                 'frac_of_measured_hbm': round(gbs / hbm_peak, 3), 'bytes_per_call': nbytes}
        del ws, g
    return res


def _graph_time_us(torch, fn_list, reps_per_graph, replays=5):
    """Mean device time (us) of one call, captured in a CUDA graph that cycles
    through ``fn_list`` (one entry per weight copy)."""
    for f in fn_list:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(reps_per_graph):
                fn_list[i % len(fn_list)]()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (replays * reps_per_graph)


def dense_ffn_probe(torch, synth, hbm_peak, tc_peak):
    """Configuration 2: dense Q4_K FFN (gate/up [14336 x 4096], down [4096 x
    14336]) at T = 1 (GEMV path) and T = 512 (tensor-core path), three weight
    copies (297 MB, > 2 x L2) cycled in a CUDA graph."""
    from localai_b200.ffn import QuantFFN
    Dm, Ff = 4096, 14336
    rng = np.random.default_rng(2)
    dev = lambda b: torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()
    raws = [synth.q4_k(rng, Ff, Dm), synth.q4_k(rng, Ff, Dm), synth.q4_k(rng, Dm, Ff)]
    ffns = []
    for _ in range(3):
        ffns.append(QuantFFN(dev(raws[0]), dev(raws[1]), dev(raws[2]), d_model=Dm, d_ff=Ff))
    wbytes = sum(len(r) for r in raws)
    res = {}
    for T in (1, 512):
        x = torch.randn(T, Dm, device='cuda')
        us = _graph_time_us(torch, [lambda f=f: f(x) for f in ffns], 30 if T == 1 else 6)
        flops = 2.0 * T * 3 * Ff * Dm
        ent = {'us_per_call': round(us, 2), 'flops': flops}
        if T == 1:
            nbytes = wbytes + 4 * (Dm + 2 * Ff + Ff + Dm)
            ent.update({'GB_s': round(nbytes / (us * 1e-6) / 1e9, 1),
                        'frac_of_measured_hbm': round(nbytes / (us * 1e-6) / 1e9 / hbm_peak, 3),
                        'bytes_per_call': nbytes, 'path': 'GEMV [gate;up] + silu*up + GEMV down'})
        else:
            ent.update({'TFLOP_s': round(flops / (us * 1e-6) / 1e12, 1),
                        'frac_of_measured_bf16': round(flops / (us * 1e-6) / 1e12 / tc_peak, 3),
                        'path': 'tcgen05 GEMM gate/up (fused SiLU*up) + GEMM down'})
        res[f'T{T}'] = ent
    del ffns
    return res


def _q8_0_device(torch, rows, cols, gen, d_sigma=0.005):
    """Synthetic Q8_0 matrix generated on the device (same distribution as
    synth.q8_0: d = fp16(|N(0, d_sigma)|), q uniform in [-127, 127])."""
    nb = rows * (cols // 32)
    d = (torch.randn(nb, device='cuda', generator=gen) * d_sigma).abs().half()
    q = torch.randint(-127, 128, (nb, 32), device='cuda', dtype=torch.int8, generator=gen)
    blocks = torch.empty((nb, 34), dtype=torch.uint8, device='cuda')
    blocks[:, 0:2] = d.view(torch.uint8).reshape(nb, 2)
    blocks[:, 2:] = q.view(torch.uint8)
    return blocks.reshape(-1)


def decode_probe(torch, hbm_peak, prompt_len=2048, new_tokens=128):
    """Configuration 4: Llama-3-8B-shaped decoder (32 layers, hidden 4096, 32
    heads / 8 KV heads, FFN 14336, vocabulary 128256), every matrix Q8_0 (8.53
    GB), greedy: a prompt of ``prompt_len`` random token ids fed through the
    captured decode step (untimed), then ``new_tokens`` timed steps."""
    from localai_b200.decoder import LlamaConfig, QuantLlama
    NL, Dm, H, KV, Ff, V = 32, 4096, 32, 8, 14336, 128256
    hd = Dm // H
    gen = torch.Generator(device='cuda')
    gen.manual_seed(4)
    ones = torch.ones(Dm, device='cuda')
    layers = []
    for _ in range(NL):
        layers.append({'attn_q': (_q8_0_device(torch, H * hd, Dm, gen), 8),
                       'attn_k': (_q8_0_device(torch, KV * hd, Dm, gen), 8),
                       'attn_v': (_q8_0_device(torch, KV * hd, Dm, gen), 8),
                       'attn_output': (_q8_0_device(torch, Dm, Dm, gen), 8),
                       'ffn_gate': (_q8_0_device(torch, Ff, Dm, gen), 8),
                       'ffn_up': (_q8_0_device(torch, Ff, Dm, gen), 8),
                       'ffn_down': (_q8_0_device(torch, Dm, Ff, gen), 8),
                       'attn_norm': ones, 'ffn_norm': ones})
    w = {'token_embd': (_q8_0_device(torch, V, Dm, gen), 8), 'output': (_q8_0_device(torch, V, Dm, gen), 8),
         'output_norm': ones, 'layers': layers}
    cfg = LlamaConfig(n_layers=NL, d_model=Dm, n_heads=H, n_kv_heads=KV, d_ff=Ff, vocab=V, rope_base=500000.0,
                      eps=1e-5, max_seq=prompt_len + new_tokens)
    model = QuantLlama(w, cfg)
    del w, layers
    wbytes = 34 * (NL * ((H * hd + 2 * KV * hd) * Dm + Dm * Dm + 2 * Ff * Dm + Dm * Ff) + 2 * V * Dm) // 32
    prompt = torch.randint(0, V, (prompt_len,), generator=torch.Generator().manual_seed(5)).tolist()
    model.reset()
    model.set_token(prompt[0])
    model.step()
    model.capture()
    model.reset()
    model.prefill(prompt[:64])                       # set-up of the prefill path (untimed)
    model.reset()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    model.prefill(prompt)
    p1.record()
    torch.cuda.synchronize()
    prefill_ms = p0.elapsed_time(p1)
    params = NL * ((H * hd + 2 * KV * hd) * Dm + Dm * Dm + 3 * Ff * Dm)
    prefill_flops = 2.0 * params * prompt_len + 4.0 * NL * H * hd * prompt_len * (prompt_len + 1) / 2
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(new_tokens):
        model.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / new_tokens
    ctx = prompt_len + new_tokens / 2
    kv_bytes = 2 * NL * ctx * KV * hd * 4
    nbytes = wbytes + kv_bytes
    res = {'decode_tokens_per_s': round(1e3 / ms, 1), 'ms_per_token': round(ms, 3),
           'GB_s': round(nbytes / (ms * 1e-3) / 1e9, 1), 'frac_of_measured_hbm': round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 3),
           'bytes_per_token': int(nbytes), 'weights_bytes': int(wbytes), 'prompt_tokens': prompt_len,
           'timed_tokens': new_tokens,
           'prefill': {'ms': round(prefill_ms, 2), 'tokens_per_s': round(prompt_len / (prefill_ms * 1e-3), 1),
                       'TFLOP_s': round(prefill_flops / (prefill_ms * 1e-3) / 1e12, 1), 'flops': prefill_flops,
                       'path': 'tcgen05 GEMMs over the prompt rows + causal attention kernel'},
           'launches_per_token': 5 + NL * 10,
           'path': 'CUDA graph of one step: per layer 4 GEMVs + 2 norms, RoPE/KV store, 2 attention kernels, SiLU*up; '
                   'every launch programmatic-dependent'}
    del model
    torch.cuda.empty_cache()
    return res


def moe_q6k_probe(torch, synth):
    """Configuration 3: Q6_K MoE, D=2048, E=16, F=1024, top-2, T = 1, 64, 4096
    (four layer copies, 330 MB of expert weights = more than twice the L2,
    cycled in a CUDA graph)."""
    from localai_b200.moe import QuantMoE
    E3, D3, F3, k3 = 16, 2048, 1024, 2
    rng = np.random.default_rng(3)
    dev = lambda b: torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()
    gu = b''.join(synth.q6_k(rng, 2 * F3, D3) for _ in range(E3))
    dn = b''.join(synth.q6_k(rng, D3, F3) for _ in range(E3))
    wr3 = torch.from_numpy(rng.normal(0, 0.02, size=(E3, D3)).astype(np.float32)).cuda()
    layers = [QuantMoE(wr3, dev(gu), dev(dn), d_model=D3, d_ff=F3, top_k=k3, ggml_type=14) for _ in range(4)]
    res = {}
    for T in (1, 64, 4096):
        h3 = torch.randn(T, D3, device='cuda')
        us = _graph_time_us(torch, [lambda L=L: L(h3) for L in layers], 20 if T < 4096 else 6)
        res[f'T{T}'] = {'us_per_call': round(us, 2), 'tokens_per_s': round(T / (us * 1e-6), 1)}
    del layers
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--cpu-tokens', type=int, default=2048, help='token sample of the CPU baseline')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-gemv', action='store_true')
    ap.add_argument('--ep-unfused', action='store_true',
                    help='N > 1, p2p: separate send kernel before the expert GEMMs instead of the '
                         'exchange fused into the gate/up GEMM')
    ap.add_argument('--transport', default='p2p', choices=['p2p', 'nccl'],
                    help='expert-parallel exchange (N > 1): NVLink peer memory or NCCL all-to-all')
    ap.add_argument('--phases', action='store_true',
                    help='N > 1, p2p: add per-rank stage times of one layer call ("ep_phases")')
    ap.add_argument('--e2e-chunks', type=str, default='1,2,3,4,6,8',
                    help='token chunk counts tried for the end-to-end leg (PCIe copies overlapped with '
                         'compute); the fastest is reported')
    ap.add_argument('--tokens', type=int, default=T_TOTAL,
                    help='tokens per layer call (16384 = the headline configuration; smaller for profiling)')
    args = ap.parse_args()
    set_tokens(args.tokens)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == 'reference':
        run_reference_arm(args)
        return

    import torch
    import torch.distributed as dist
    from localai_b200 import _lib, ops, synth
    from localai_b200.moe import QuantMoE
    from localai_b200.ep import EPMoE, lpt_placement

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local_rank)
    dev = torch.device('cuda', local_rank)
    if world > 1:
        dist.init_process_group('nccl', timeout=timedelta(seconds=300), device_id=dev)
    lib = _lib.load()
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    hbm_peak = float(peaks.get('hbm_gbs', 6650.0))
    tc_burst = float(peaks.get('bf16_tflops', 1590.0))
    peak_src = 'measured' if peaks else 'fallback'

    wr = torch.from_numpy(router_weights()).to(dev)
    bias = torch.from_numpy(zipf_bias()).to(dev)
    T_loc = T_TOTAL // world
    t0, t1 = rank * T_loc, (rank + 1) * T_loc
    h = hidden_states(torch, dev, t0, t1)

    # expert placement: LPT on the routing loads of a calibration batch (same
    # distribution, different seed from the timed tokens; setup, untimed)
    if world > 1:
        probe = QuantMoE.__new__(QuantMoE)
        probe.E, probe.D, probe.k, probe.renorm, probe.sel_bias = E, D, K_TOP, 1, None
        probe.router_w, probe.router_bias, probe.lib = wr, bias, lib
        _, ids_all, _ = probe.route(hidden_states(torch, dev, 0, T_TOTAL, seed=4242))
        loads = torch.bincount(ids_all.reshape(-1).long(), minlength=E).cpu().numpy()
        owner, local = lpt_placement(loads, world)
        mine = [int(e) for e in np.nonzero(owner == rank)[0]]
    else:
        owner = local = None
        mine = list(range(E))
    parts = [expert_weights(e) for e in mine]
    gate_up = torch.frombuffer(bytearray(b''.join(p[0] for p in parts)), dtype=torch.uint8).to(dev)
    down = torch.frombuffer(bytearray(b''.join(p[1] for p in parts)), dtype=torch.uint8).to(dev)
    del parts
    layer = QuantMoE(wr, gate_up, down, d_model=D, d_ff=F, top_k=K_TOP, router_bias=bias, renormalize=True,
                     local_experts=len(mine))
    step = (EPMoE(layer, owner, local, transport=args.transport, max_tokens=T_loc, fused=not args.ep_unfused)
            if world > 1 else layer)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # clock sampling starts before the warm-up so that nvidia-smi's own start-up
    # does not fall into the timed region
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(1.0)
    barrier()
    # warm-up: W steps (more would push the part into its power-capped
    # regime before the timed region; it idles at full clock)
    for _ in range(args.warmup):
        step(h)
    warm_steps = args.warmup
    torch.cuda.synchronize()
    ops.check_device_error()

    # ---- timed region (device-resident inputs)
    barrier()
    torch.cuda.synchronize()
    n0 = lib.b200q_launch_count()
    g0_launches = getattr(step, 'graph_launches', 0)
    t_start = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        y = step(h)
    e1.record()
    torch.cuda.synchronize()
    t_end = time.time()
    launches = lib.b200q_launch_count() - n0 + getattr(step, 'graph_launches', 0) - g0_launches
    barrier()
    clocks = sampler.stop(t_start, t_end) if sampler else None
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    value = T_TOTAL / (ms * 1e-3)

    # ---- end to end through the public API: host (pinned) input and output;
    # forward_host overlaps the PCIe copies with the layer computation
    h_host = h.cpu().pin_memory()
    y_host = torch.empty((T_loc, D), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(args.steps, 5))
    # the chunk count is the caller's choice in the public API; more chunks
    # hide more of the PCIe time but pay the layer's fixed per-call costs more
    # often (expert parallelism: a count exchange per call), so a few are tried
    e2e_trials = {}
    for nch in sorted({max(1, min(int(c), T_loc)) for c in args.e2e_chunks.split(',')}):
        step.forward_host(h_host, y_host, chunks=nch)              # warm the extra streams/buffers and graphs
        barrier()
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record()
        for _ in range(e2e_steps):
            step.forward_host(h_host, y_host, chunks=nch)
        e3.record()
        torch.cuda.synchronize()
        ms_e2e = torch.tensor([e2.elapsed_time(e3) / e2e_steps], device=dev)
        if world > 1:
            dist.all_reduce(ms_e2e, op=dist.ReduceOp.MAX)
        e2e_trials[nch] = T_TOTAL / (float(ms_e2e.item()) * 1e-3)
    e2e_chunks = max(e2e_trials, key=e2e_trials.get)
    e2e_value = e2e_trials[e2e_chunks]

    # ---- dominant kernel: the gate/up grouped GEMM, timed alone on this rank's experts
    _, ids, w = layer.route(h)
    if world > 1:
        ids = step.virt[ids.long()]
    offsets, slot_of, _, slot_w, xperm = layer.dispatch(h, ids, w)
    slots = xperm.shape[0]
    act = torch.empty((slots, F), dtype=torch.bfloat16, device=dev)
    gemm_reps = 5
    n_groups = E if world == 1 else E    # virtual-expert grouping of this rank's own tokens
    gu_all = gate_up if world == 1 else None
    roof = None
    if world == 1:
        for _ in range(2):
            ops.gemm_q4k(xperm, gu_all, offsets, k=D, n_feat=F, w_rows_per_group=2 * F, up_offset=F, act=act)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(gemm_reps):
            ops.gemm_q4k(xperm, gu_all, offsets, k=D, n_feat=F, w_rows_per_group=2 * F, up_offset=F, act=act)
        g1.record()
        torch.cuda.synchronize()
        gemm_ms = g0.elapsed_time(g1) / gemm_reps
        flops = 2.0 * slots * (2 * F) * D
        achieved = flops / (gemm_ms * 1e-3) / 1e12
        # DRAM bytes of one full-size gate/up launch, from the committed ncu
        # capture (only meaningful for the full token count)
        traffic = None
        if PROFILE_TRAFFIC.exists() and T_TOTAL == T_HEADLINE:
            for line in PROFILE_TRAFFIC.read_text().splitlines():
                if line.startswith('traffic_bytes_per_launch:'):
                    traffic = float(line.split(':', 1)[1].split()[0])
        algo_bytes = gate_up.numel() + slots * D * 2 + slots * F * 2
        # the down GEMM alone as well (same kernel, plain bf16 epilogue, K = 1408)
        out_dn = torch.empty((slots, D), dtype=torch.bfloat16, device=dev)
        down_call = lambda: ops.gemm_q4k(act, down, offsets, k=F, n_feat=D, w_rows_per_group=D, out=out_dn,
                                         row_scale=slot_w)
        down_call()
        torch.cuda.synchronize()
        g0.record()
        for _ in range(gemm_reps):
            down_call()
        g1.record()
        torch.cuda.synchronize()
        down_ms = g0.elapsed_time(g1) / gemm_reps
        down_flops = 2.0 * slots * D * F
        roof = {'kernel': 'tc_gemm_q4k_kernel (gate/up, fused SiLU*up)', 'bound': 'tensor',
                'achieved': round(achieved, 1), 'peak': tc_burst, 'unit': 'TFLOP/s',
                'frac': round(achieved / tc_burst, 3), 'traffic': traffic, 'algorithmic_bytes': int(algo_bytes),
                'peak_source': f'{peak_src} bf16 (burst; kernel timed alone)',
                'flops_per_launch': flops, 'ms_per_launch': round(gemm_ms, 4),
                'down_gemm': {'ms_per_launch': round(down_ms, 4), 'flops_per_launch': down_flops,
                              'achieved': round(down_flops / (down_ms * 1e-3) / 1e12, 1)}}

    phases = None
    if world > 1 and args.phases and args.transport == 'p2p':
        mine_ph = step.phase_times(h)
        allp = [None] * world
        dist.all_gather_object(allp, mine_ph)
        phases = {f'rank{r}': p for r, p in enumerate(allp)}
    gemv = ffn2 = moe3 = dec4 = None
    if rank == 0 and not args.no_gemv and world == 1:
        gemv = gemv_probe(torch, ops, synth, hbm_peak)
        ffn2 = dense_ffn_probe(torch, synth, hbm_peak, tc_burst)
        moe3 = moe_q6k_probe(torch, synth)
        dec4 = decode_probe(torch, hbm_peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, kind, cores, dt = cpu_reference_moe(args.cpu_tokens)
        cpu = {'value': v, 'unit': 'tokens/s', 'cores': cores, 'kind': kind,
               'sample': f'{args.cpu_tokens} of {T_TOTAL} tokens (same layer shapes and routing), {dt:.1f} s'}
        if not args.no_gemv:
            cpu['other_configs'] = cpu_reference_extras()

    if rank == 0:
        line = {'metric': METRIC, 'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps,
                'warmup': warm_steps, 'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'strong',
                'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
                'config': {'workload': WORKLOAD, 'hidden': D, 'experts': E, 'intermediate': F, 'top_k': K_TOP,
                           'tokens': T_TOTAL, 'weights': 'Q4_K', 'router': 'f32 + Zipf(1.1) bias',
                           'parallelism': f'ep{world}' if world > 1 else 'single',
                           'ep_transport': (args.transport + ('' if args.ep_unfused or args.transport != 'p2p'
                                                              else ', exchange fused into the gate/up GEMM'))
                                           if world > 1 else None,
                           'l2': 'inputs larger than L2 (641 MB expert weights, 256 MB hidden states)'},
                'roofline': roof, 'cpu_baseline': cpu,
                'e2e': {'value': e2e_value, 'unit': 'tokens/s', 'h2d_bytes_per_step': T_TOTAL * D * 4,
                        'd2h_bytes_per_step': T_TOTAL * D * 4, 'chunks': e2e_chunks,
                        'chunk_trials': {str(c): round(v, 1) for c, v in e2e_trials.items()},
                        'api': 'EPMoE.forward_host' if world > 1 else 'QuantMoE.forward_host'},
                'gpu_launches': int(launches), 'clocks': clocks, 'gemv': gemv,
                'config2_dense_ffn_q4k': ffn2, 'config3_moe_q6k': moe3, 'config4_decode_q8_0': dec4,
                'ep_phases': phases,
                'flops_per_step': algorithmic_flops(T_TOTAL * K_TOP)}
        print(json.dumps(line), flush=True)
    if world > 1:
        if hasattr(step, 'close'):
            step.close()
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
