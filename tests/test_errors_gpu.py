"""GPU tests of the error paths: bad indices and timed-out waits are reported
through the device error word and touch no memory outside the buffers.

* dispatch with expert ids outside [0, E): those pairs get slot -1 and no
  slot, every other pair is dispatched exactly as without them, the gather
  reads only assigned slots, the combine skips the unassigned ones, and
  ``b200q_check_device_error`` reports ERR_BAD_INDEX (2) once;
* prefill attention at a position past the cache writes nothing and reports 2;
* an expert-parallel wait on a flag nobody raises (one rank, 0.2 s limit)
  returns and reports ERR_WAIT_TIMEOUT (1); the context stays usable.
"""
import ctypes

import numpy as np
import pytest
import torch

from localai_b200 import _lib

pytestmark = pytest.mark.gpu

ERR_WAIT_TIMEOUT, ERR_BAD_INDEX = 1, 2


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dispatch(lib, ids, w, h, E):
    T, k = ids.shape
    D, dev, S = h.shape[1], ids.device, ids.numel()
    nblk = lib.b200q_moe_num_blocks(T)
    scratch = torch.empty((2, nblk * E), dtype=torch.int32, device=dev)
    offsets = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    slot_of = torch.full((S,), -7, dtype=torch.int32, device=dev)
    token_of = torch.full((S,), -7, dtype=torch.int32, device=dev)
    slot_w = torch.zeros((S,), dtype=torch.float32, device=dev)
    xperm = torch.zeros((S, D), dtype=torch.bfloat16, device=dev)
    _lib.check(lib.b200q_moe_dispatch_dev(ids.data_ptr(), w.data_ptr(), T, k, E, h.data_ptr(), D,
                                          scratch[0].data_ptr(), scratch[1].data_ptr(), offsets.data_ptr(),
                                          slot_of.data_ptr(), token_of.data_ptr(), slot_w.data_ptr(),
                                          xperm.data_ptr(), _stream()))
    return offsets, slot_of, token_of, slot_w, xperm


def test_dispatch_and_combine_with_bad_expert_ids():
    lib = _lib.load()
    torch.cuda.set_device(0)
    assert lib.b200q_check_device_error() == 0
    T, k, E, D = 600, 4, 16, 256
    g = torch.Generator(device='cuda')
    g.manual_seed(7)
    ids = torch.topk(torch.rand((T, E), generator=g, device='cuda'), k, dim=1).indices.to(torch.int32)
    w = torch.rand((T, k), generator=g, device='cuda')
    h = torch.randn((T, D), generator=g, device='cuda')
    bad = ids.clone()
    bad[3, 1] = E            # one past the end
    bad[250, 0] = -1
    bad[599, 3] = 1 << 20
    n_bad = 3
    offsets, slot_of, token_of, slot_w, xperm = _dispatch(lib, bad.contiguous(), w, h, E)
    assert lib.b200q_check_device_error() == ERR_BAD_INDEX
    assert lib.b200q_check_device_error() == 0          # read and cleared
    # reference: the same dispatch with the bad pairs' ids replaced by a dropped marker, on the host
    ids_h, w_h = bad.cpu().numpy(), w.cpu().numpy()
    valid = (ids_h >= 0) & (ids_h < E)
    assert int(offsets[-1]) == T * k - n_bad
    so = slot_of.cpu().numpy().reshape(T, k)
    assert np.all(so[~valid] == -1)
    counts = np.bincount(ids_h[valid], minlength=E)
    assert np.array_equal(np.diff(offsets.cpu().numpy()), counts)
    # stable order inside each expert, weights and gathered rows of every assigned slot
    tok = token_of.cpu().numpy()
    sw = slot_w.cpu().numpy()
    hb = h.to(torch.bfloat16).cpu()
    xp = xperm.cpu()
    order = [(e, t, j) for t in range(T) for j in range(k) if valid[t, j] for e in [ids_h[t, j]]]
    order.sort(key=lambda r: (r[0], r[1], r[2]))
    for slot, (e, t, j) in enumerate(order):
        assert so[t, j] == slot and tok[slot] == t and sw[slot] == w_h[t, j]
    assert torch.equal(xp[:T * k - n_bad], hb[torch.from_numpy(tok[:T * k - n_bad]).long()])
    # combine: unassigned slots add nothing
    out = torch.randn((T * k, D), generator=g, device='cuda')
    y = torch.empty((T, D), device='cuda')
    _lib.check(lib.b200q_moe_combine_dev(out.data_ptr(), 0, slot_of.data_ptr(), slot_w.data_ptr(), T, k, D,
                                         y.data_ptr(), _stream()))
    torch.cuda.synchronize()
    o_h = out.cpu().numpy()
    ref = np.zeros((T, D), np.float32)
    for t in range(T):
        for j in range(k):
            if so[t, j] >= 0:
                ref[t] += sw[so[t, j]] * o_h[so[t, j]]
    np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    assert lib.b200q_check_device_error() == 0


def test_gather_f32_rejects_bad_token():
    lib = _lib.load()
    T, D, S = 10, 64, 5
    h = torch.randn((T, D), device='cuda')
    token_of = torch.tensor([0, 9, 10, -3, 4], dtype=torch.int32, device='cuda')
    out = torch.full((S, D), 7.0, device='cuda')
    _lib.check(lib.b200q_moe_gather_f32_dev(h.data_ptr(), T, token_of.data_ptr(), S, D, out.data_ptr(), _stream()))
    assert lib.b200q_check_device_error() == ERR_BAD_INDEX
    assert torch.equal(out[0], h[0]) and torch.equal(out[1], h[9]) and torch.equal(out[4], h[4])
    assert torch.all(out[2] == 7.0) and torch.all(out[3] == 7.0)


def test_attn_prefill_position_out_of_range():
    lib = _lib.load()
    H, KV, hd, max_seq, T = 4, 2, 64, 8, 4
    qkv = torch.randn((T, (H + 2 * KV) * hd), device='cuda')
    kc = torch.randn((max_seq, KV, hd), device='cuda')
    vc = torch.randn((max_seq, KV, hd), device='cuda')
    out = torch.full((T, H * hd), 3.0, dtype=torch.bfloat16, device='cuda')
    for p in (5, -1):                      # 5 + 4 > 8, and a negative position
        pos = torch.tensor([p], dtype=torch.int32, device='cuda')
        _lib.check(lib.b200q_attn_prefill_dev(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), T, H,
                                              KV, hd, max_seq, out.data_ptr(), _stream()))
        assert lib.b200q_check_device_error() == ERR_BAD_INDEX
        assert torch.all(out == 3.0)
    # a valid position still works afterwards
    pos = torch.tensor([4], dtype=torch.int32, device='cuda')
    _lib.check(lib.b200q_attn_prefill_dev(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), T, H,
                                          KV, hd, max_seq, out.data_ptr(), _stream()))
    assert lib.b200q_check_device_error() == 0
    assert not torch.any(out == 3.0)


def test_ep_wait_times_out_and_reports():
    """One rank, a return flag nobody raises: the bounded wait gives up after
    the (shortened) limit, the combine still runs on in-bounds rows, the error
    word says ERR_WAIT_TIMEOUT, and later work on the device succeeds."""
    lib = _lib.load()
    torch.cuda.set_device(0)
    D = 64
    ep = ctypes.c_void_p()
    _lib.check(lib.b200q_ep_create(1, 0, 1, D, 4, 4, ctypes.byref(ep)))
    try:
        handle = ctypes.create_string_buffer(lib.b200q_ep_handle_bytes())
        _lib.check(lib.b200q_ep_handle(ep, handle))
        _lib.check(lib.b200q_ep_open(ep, handle))
        lib.b200q_ep_set_wait_limit_ns(200_000_000)
        slot_of = torch.zeros(1, dtype=torch.int32, device='cuda')
        slot_w = torch.ones(1, device='cuda')
        y = torch.empty((1, D), device='cuda')
        torch.cuda.synchronize()
        _lib.check(lib.b200q_ep_combine_dev(ep, slot_of.data_ptr(), slot_w.data_ptr(), 1, 1, y.data_ptr(), 7,
                                            _stream()))
        assert lib.b200q_check_device_error() == ERR_WAIT_TIMEOUT
        x = torch.arange(10, device='cuda', dtype=torch.float32)
        assert float((x * 2).sum()) == 90.0
        assert lib.b200q_check_device_error() == 0
    finally:
        lib.b200q_ep_set_wait_limit_ns(0)
        _lib.check(lib.b200q_ep_destroy(ep))
