"""Generate tests/golden/zaya_gguf_golden.npz: the reference's own
``ZayaModel._moe`` (engine/zaya.py:139-175,274-307) reading one MoE layer from
a seeded GGUF file through its own ``GGUFFile``: the router matrices with
their ``.bias`` tensors (added by ``LlamaModel.mat``, engine/model.py:73-79),
and the packed expert tensors ``ffn_gate_up_exps`` [E, 2F, D] (Q4_K) and
``ffn_down_exps`` [E, D, F] (Q6_K) that ``_expert_matvec`` slices one expert
at a time.

The model object is the reference class with only the fields ``_moe`` and
its helpers read (``gguf``, ``n_experts``, ``eps``, the weight and expert
caches); its native kernels are switched off, so every product is the exact
dequantise-then-f32 path.  The fixture keeps the file's SHA-256 (tests
rebuild the file with ``build_file``), the inputs, the reference's outputs,
router states and chosen routes (E = the skip route).

    python tests/golden/make_zaya_gguf_golden.py <reference checkout>
"""
import hashlib
import shutil
import sys
import tempfile
from collections import OrderedDict
from pathlib import Path

import numpy as np

E, D, F, R, R2, R3, T, LAYER = 8, 512, 256, 256, 128, 64, 24, 1


def build_file(path):
    """Write the seeded one-layer ZAYA MoE GGUF file to ``path``."""
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from localai_b200 import synth
    from localai_b200.gguf import write_gguf
    rng = np.random.default_rng(604)
    f = lambda *s, sc=1.0: rng.normal(0, sc, size=s).astype(np.float32)
    f32 = lambda a: (a.tobytes(), 0, a.shape)
    p = f'blk.{LAYER}.'
    t = {p + 'ffn_gate_inp.weight': f32(f(R, D, sc=D ** -0.5)), p + 'ffn_gate_inp.bias': f32(f(R, sc=0.1)),
         p + 'ffn_gate.weight': f32(f(R2, R, sc=R ** -0.5)), p + 'ffn_gate.bias': f32(f(R2, sc=0.1)),
         p + 'zaya_router_mlp2.weight': f32(f(R3, R2, sc=R2 ** -0.5)),
         p + 'zaya_router_mlp2.bias': f32(f(R3, sc=0.1)),
         p + 'zaya_router_mlp4.weight': f32(f(E + 1, R3, sc=4 * R3 ** -0.5)),
         p + 'ffn_norm.weight': f32((1 + f(R, sc=0.1)).astype(np.float32)),
         p + 'zaya_router_eda.weight': f32(f(R, sc=0.5)),
         # well-separated route biases: the chosen expert is far from a tie
         p + 'zaya_router_biases.weight': f32(np.concatenate([f(E, sc=0.3), [0.05]]).astype(np.float32)),
         p + 'ffn_gate_up_exps.weight': (b''.join(synth.q4_k(rng, 2 * F, D) for _ in range(E)), 12, (E, 2 * F, D)),
         p + 'ffn_down_exps.weight': (b''.join(synth.q6_k(rng, D, F) for _ in range(E)), 14, (E, D, F))}
    write_gguf(path, {'general.architecture': 'zaya', 'zaya.expert_count': E}, t)


def inputs():
    rng = np.random.default_rng(605)
    H = rng.normal(size=(T, D)).astype(np.float32)
    P = rng.normal(size=(T, R)).astype(np.float32)
    return H, P


def main(ref_root):
    tmp = Path(tempfile.mkdtemp())
    shutil.copytree(Path(ref_root) / 'engine', tmp / 'engine')
    sys.path.insert(0, str(tmp))
    import engine.native_quant as nq                                 # noqa: E402
    nq._LIB, nq._TRIED = None, True                                  # exact f32 products, no native kernels
    from engine.gguf_parser import GGUFFile                          # noqa: E402
    from engine.zaya import ZayaModel                                # noqa: E402

    path = tmp / 'zaya.gguf'
    build_file(path)
    chosen = []

    class Recording(ZayaModel):
        def _expert_matvec(self, name, expert, x):
            if name.endswith('ffn_gate_up_exps.weight'):
                chosen[-1] = int(expert)
            return super()._expert_matvec(name, expert, x)

    H, P = inputs()
    Y = np.empty((T, D), np.float32)
    S = np.empty((T, R), np.float32)
    with GGUFFile(path) as g:
        m = Recording.__new__(Recording)
        m.gguf, m.n_experts, m.eps = g, E, 1e-5
        m._weights, m._expert_cache, m._expert_cache_limit = {}, OrderedDict(), 4
        for t in range(T):
            chosen.append(E)                                         # the skip route unless an expert runs
            y, s = m._moe(LAYER, H[t], P[t] if t % 3 else None)
            Y[t], S[t] = y, s
    dst = Path(__file__).resolve().parent / 'zaya_gguf_golden.npz'
    np.savez_compressed(dst, H=H, P=P, Y=Y, S=S, route=np.asarray(chosen, np.int32),
                        sha256=np.asarray(hashlib.sha256(path.read_bytes()).hexdigest()))
    print('routes', chosen)
    print(f'wrote {dst}')


if __name__ == '__main__':
    main(sys.argv[1])
