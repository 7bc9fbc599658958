"""GPU tests of the grouped decode GEMV (MoE experts at small batch) and of
QuantMoE's decode path built on it.

Each group g multiplies its own weight matrix with its own token rows
[off[g], off[g+1]); empty groups read nothing.  Bar: the float64 oracle,
normwise <= 1e-3 per group (f32 accumulation, as the single GEMV).
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200 import _lib, ops, synth
from localai_b200.moe import QuantMoE

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('t,rows,cols,pad', [(12, 256, 1024, 0), (14, 384, 1024, 8), (8, 128, 512, 0),
                                             (12, 200, 4096, 0)])
def test_grouped_gemv(t, rows, cols, pad):
    rng = np.random.default_rng(t + rows + cols)
    G = 6
    sizes = [2, 0, 1, 5, 0, 3] if cols <= 1024 else [2, 0, 1, 3, 0, 2]     # within the per-launch token cap
    raws = [synth.make(rng, t, rows, cols) for _ in range(G)]
    rb = o.row_bytes(t, cols)
    stride = rb + pad
    w = np.zeros((G, rows, stride), np.uint8)
    for g in range(G):
        w[g, :, :rb] = np.frombuffer(raws[g], np.uint8).reshape(rows, rb)
    wd = torch.from_numpy(w.reshape(-1)).cuda()
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    S = int(off[-1])
    x = rng.normal(size=(S, cols)).astype(np.float32)
    y = torch.full((S, rows), float('nan'), device='cuda')
    offd = torch.from_numpy(off).cuda()          # kept alive until the kernel has run
    xd = torch.from_numpy(x).cuda()
    lib = _lib.load()
    assert S <= lib.b200q_gemv_grouped_max_tokens(t, cols)
    _lib.check(lib.b200q_gemv_grouped_dev(t, wd.data_ptr(), rows * stride, stride if pad else 0, G, offd.data_ptr(),
                                          xd.data_ptr(), y.data_ptr(), rows, rows, cols, S, S, 4,
                                          torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ops.check_device_error()
    yn = y.cpu().numpy()
    for g in range(G):
        a, b = off[g], off[g + 1]
        if a == b:
            continue
        ref = o.matmul_f64(raws[g], t, rows, cols, x[a:b])
        assert o.normwise_rel_err(yn[a:b], ref) < 1e-3, g


def test_grouped_gemv_rejects_too_many_tokens():
    lib = _lib.load()
    cap = lib.b200q_gemv_grouped_max_tokens(12, 4096)
    assert 1 <= cap <= 64
    w = torch.zeros(2304 * 8, dtype=torch.uint8, device='cuda')
    off = torch.tensor([0, cap + 1], dtype=torch.int32, device='cuda')
    x = torch.zeros((cap + 1, 4096), device='cuda')
    y = torch.zeros((cap + 1, 8), device='cuda')
    st = lib.b200q_gemv_grouped_dev(12, w.data_ptr(), 0, 0, 1, off.data_ptr(), x.data_ptr(), y.data_ptr(), 8, 8,
                                    4096, cap + 1, cap + 1, 1, torch.cuda.current_stream().cuda_stream)
    assert st == -1


def test_grouped_gemv_bad_offsets_are_reported():
    """Offsets outside x/y are refused on the device: no access, error word set."""
    lib = _lib.load()
    w = torch.zeros(2304 * 8, dtype=torch.uint8, device='cuda')
    off = torch.tensor([0, 3, 1000], dtype=torch.int32, device='cuda')      # group 1 ends past the 4 rows
    x = torch.zeros((4, 4096), device='cuda')
    y = torch.zeros((4, 8), device='cuda')
    st = lib.b200q_gemv_grouped_dev(12, w.data_ptr(), 0, 0, 2, off.data_ptr(), x.data_ptr(), y.data_ptr(), 8, 8,
                                    4096, 4, 4, 2, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    with pytest.raises(_lib.B200QError):
        ops.check_device_error()


@pytest.mark.parametrize('E,D,F,k,T,t', [(8, 512, 128, 2, 1, 12), (16, 1024, 192, 4, 3, 12),
                                         (16, 2048, 1024, 2, 1, 14), (8, 512, 256, 2, 4, 8)])
def test_moe_decode_path_matches_oracle(E, D, F, k, T, t):
    """QuantMoE.forward at decode-sized batches takes the grouped-GEMV path:
    f32 accumulation, so the 1e-3 bar of the GEMV applies."""
    rng = np.random.default_rng(E * D + T)
    blk = 32 if t == 8 else 256
    F_pad = (F + blk - 1) // blk * blk
    gen = {12: synth.q4_k, 14: synth.q6_k, 8: synth.q8_0}[t]
    gate_up = [gen(rng, 2 * F, D) for _ in range(E)]
    if t == 12:
        down = [synth.q4_k(rng, D, F_pad, zero_tail_cols=F_pad - F) for _ in range(E)]
    else:
        assert F_pad == F
        down = [gen(rng, D, F) for _ in range(E)]
    wr = rng.normal(0, D ** -0.5, size=(E, D)).astype(np.float32)
    cat = lambda parts: torch.frombuffer(bytearray(b''.join(parts)), dtype=torch.uint8).cuda()
    layer = QuantMoE(torch.from_numpy(wr).cuda(), cat(gate_up), cat(down), d_model=D, d_ff=F, top_k=k, ggml_type=t)
    assert T * k <= layer.small_slots
    h = rng.normal(size=(T, D)).astype(np.float32)
    hd = torch.from_numpy(h).cuda()
    y = layer(hd)
    torch.cuda.synchronize()
    ops.check_device_error()
    _, ids, w = layer.route(hd)
    ref = o.moe_forward_f64(h, ids.cpu().numpy(), w.cpu().numpy(), list(zip(gate_up, down)), t, t, D, F, F_pad)
    assert o.normwise_rel_err(y.cpu().numpy(), ref) < 1e-3
