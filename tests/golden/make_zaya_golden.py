"""Generate tests/golden/zaya_moe_golden.npz by running the reference's own
``ZayaModel._moe`` (engine/zaya.py:274-307) on a stub model.

The stub supplies exactly what the method touches: ``_matvec`` (a plain f32
``W @ x (+ b)``, standing in for ``LlamaModel.mat`` on unquantised tensors),
``w``, ``gguf.tensors``, ``norm``, ``eps``, ``n_experts`` and an
``_expert_matvec`` over f32 expert matrices (the quantised expert path is
pinned separately by the dequant fixtures).  The fixture therefore pins the
router chain, the biased top-1 choice, the unbiased weighting and the skip
route.

Run in a checkout next to the reference sources (not on the GPU box):
    python tests/golden/make_zaya_golden.py /path/to/reference
"""
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np


def main(ref_root):
    tmp = Path(tempfile.mkdtemp())
    shutil.copytree(Path(ref_root) / 'engine', tmp / 'engine')      # numba caches write next to the sources
    sys.path.insert(0, str(tmp))
    from engine.zaya import ZayaModel                                 # noqa: E402
    from engine.model import LlamaModel                               # noqa: E402

    rng = np.random.default_rng(2024)
    E, D, R, R2, R3, F = 4, 64, 32, 24, 16, 20
    f = lambda *s, sc=1.0: rng.normal(0, sc, size=s).astype(np.float32)
    W = {'blk.1.ffn_gate_inp.weight': f(R, D, sc=D ** -0.5), 'blk.1.ffn_gate.weight': f(R2, R, sc=R ** -0.5),
         'blk.1.zaya_router_mlp2.weight': f(R3, R2, sc=R2 ** -0.5),
         'blk.1.zaya_router_mlp4.weight': f(E + 1, R3, sc=2 * R3 ** -0.5)}
    B = {'blk.1.ffn_gate_inp.weight': f(R, sc=0.1)}
    vec = {'blk.1.ffn_norm.weight': (1 + f(R, sc=0.1)).astype(np.float32),
           'blk.1.zaya_router_eda.weight': f(R, sc=0.5),
           'blk.1.zaya_router_biases.weight': np.concatenate([f(E, sc=0.02), [0.06]]).astype(np.float32)}
    gu = f(E, 2 * F, D, sc=D ** -0.5)
    dn = f(E, D, F, sc=F ** -0.5)

    class Stub:
        n_experts = E
        eps = 1e-5
        norm = staticmethod(LlamaModel.norm)
        _gelu = staticmethod(ZayaModel._gelu)

        class gguf:
            tensors = dict.fromkeys(list(W) + list(vec))

        def _matvec(self, name, x):
            y = W[name] @ np.asarray(x, np.float32)
            return (y + B[name]).astype(np.float32) if name in B else y.astype(np.float32)

        def w(self, name):
            return vec[name]

        def _expert_matvec(self, name, expert, x):
            m = gu[expert] if name.endswith('ffn_gate_up_exps.weight') else dn[expert]
            return (m @ np.asarray(x, np.float32)).astype(np.float32)

    stub = Stub()
    T = 48
    H = f(T, D)
    P = f(T, R)
    Y = np.empty((T, D), np.float32)
    S = np.empty((T, R), np.float32)
    for t in range(T):
        y, s = ZayaModel._moe(stub, 1, H[t], P[t] if t % 3 else None)
        Y[t], S[t] = y, s
    out = Path(__file__).resolve().parent / 'zaya_moe_golden.npz'
    np.savez_compressed(out, H=H, P=P, Y=Y, S=S, gu=gu, dn=dn, eps=np.float32(1e-5),
                        **{k.split('.', 2)[2].replace('.', '_'): v for k, v in {**W, **vec}.items()},
                        b_in=B['blk.1.ffn_gate_inp.weight'])
    print('wrote', out)


if __name__ == '__main__':
    if len(sys.argv) != 2:
        sys.exit('usage: make_zaya_golden.py <reference checkout>')
    main(sys.argv[1])
