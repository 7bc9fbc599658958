"""GPU tests of the dense quantised FFN (engine/model.py:161-166):
y = down(silu(gate x) * up x) against the float64 oracle.

Decode path (GEMV, f32 accumulation): normwise <= 1e-3.  Prefill path
(tensor cores, bf16 operands): normwise <= 1e-2.  Types follow common GGUF
mixes: all Q4_K, Q4_K with a Q6_K down projection (Q4_K_M style), all Q8_0.
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import synth
from localai_b200.ffn import QuantFFN

pytestmark = pytest.mark.gpu

GEN = {12: synth.q4_k, 14: synth.q6_k, 8: synth.q8_0}


def ffn_ref(x, gate, up, down, t, t_dn, D, F):
    g = o.matmul_f64(gate, t, F, D, x)
    u = o.matmul_f64(up, t, F, D, x)
    return o.matmul_f64(down, t_dn, D, F, o.silu(g) * u)


@pytest.mark.parametrize('t,t_dn', [(12, 12), (12, 14), (8, 8)])
@pytest.mark.parametrize('T', [1, 5, 16, 17, 300])
def test_dense_ffn(t, t_dn, T):
    D, F = 1024, 2816
    rng = np.random.default_rng(t * 1000 + t_dn * 10 + T)
    gate, up = GEN[t](rng, F, D), GEN[t](rng, F, D)
    down = GEN[t_dn](rng, D, F)
    dev = lambda b: torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()
    ffn = QuantFFN(dev(gate), dev(up), dev(down), d_model=D, d_ff=F, ggml_type=t, down_type=t_dn)
    x = rng.normal(size=(T, D)).astype(np.float32)
    y = ffn(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    ref = ffn_ref(x, gate, up, down, t, t_dn, D, F)
    bar = 1e-3 if T <= ffn.gemv_max_tokens else 1e-2
    assert o.normwise_rel_err(y.cpu().numpy(), ref) < bar


def test_dense_ffn_vector_input():
    D, F = 512, 1024
    rng = np.random.default_rng(9)
    gate, up, down = synth.q4_k(rng, F, D), synth.q4_k(rng, F, D), synth.q4_k(rng, D, F)
    dev = lambda b: torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()
    ffn = QuantFFN(dev(gate), dev(up), dev(down), d_model=D, d_ff=F)
    x = rng.normal(size=D).astype(np.float32)
    y = ffn(torch.from_numpy(x).cuda())
    assert y.shape == (D,)
    ref = ffn_ref(x[None], gate, up, down, 12, 12, D, F)[0]
    assert o.normwise_rel_err(y.cpu().numpy(), ref) < 1e-3
