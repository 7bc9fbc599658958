"""The allocation-free MoE dispatch entry point (collected last on purpose).

``b200q_moe_dispatch_noalloc_dev`` serves callers that cannot allocate device
memory -- a plugin living inside a host framework whose memory pool owns the
device budget, or a latency-critical loop that cannot afford cudaMalloc's
implicit synchronisation.  It keeps the counting-sort scratch in a static
device array instead of caller buffers.  This test calls it through the C ABI
and checks that it produces exactly what the regular dispatch produces (the
dispatch is integer bookkeeping plus a bf16 gather, so the bar is bit
equality), on two calls in a row with different routings, so a stale array
from the first call would show up in the second.
"""
import numpy as np
import pytest
import torch

from localai_b200 import _lib

pytestmark = pytest.mark.gpu


def _dispatch(lib, ids, w, h, E, noalloc):
    T, k = ids.shape
    D = h.shape[1]
    dev = ids.device
    S = T * k
    offsets = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    slot_of = torch.full((S,), -7, dtype=torch.int32, device=dev)
    token_of = torch.full((S,), -7, dtype=torch.int32, device=dev)
    slot_w = torch.full((S,), -7.0, dtype=torch.float32, device=dev)
    xperm = torch.zeros((S, D), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        st = lib.b200q_moe_dispatch_noalloc_dev(ids.data_ptr(), w.data_ptr(), T, k, E, h.data_ptr(), D,
                                                offsets.data_ptr(), slot_of.data_ptr(), token_of.data_ptr(),
                                                slot_w.data_ptr(), xperm.data_ptr(), stream)
    else:
        nblk = lib.b200q_moe_num_blocks(T)
        scratch = torch.empty((2, nblk * E), dtype=torch.int32, device=dev)
        st = lib.b200q_moe_dispatch_dev(ids.data_ptr(), w.data_ptr(), T, k, E, h.data_ptr(), D,
                                        scratch[0].data_ptr(), scratch[1].data_ptr(), offsets.data_ptr(),
                                        slot_of.data_ptr(), token_of.data_ptr(), slot_w.data_ptr(),
                                        xperm.data_ptr(), stream)
    _lib.check(st)
    torch.cuda.synchronize()
    return offsets, slot_of, token_of, slot_w, xperm


def test_noalloc_dispatch_matches_regular_dispatch_twice():
    lib = _lib.load()
    torch.cuda.set_device(0)
    for call, (T, k, E, D) in enumerate([(3000, 8, 64, 256), (777, 4, 16, 512)]):
        g = torch.Generator(device='cuda')
        g.manual_seed(100 + call)
        scores = torch.rand((T, E), generator=g, device='cuda')
        ids = torch.topk(scores, k, dim=1).indices.to(torch.int32).contiguous()
        w = torch.rand((T, k), generator=g, device='cuda')
        h = torch.randn((T, D), generator=g, device='cuda')
        ref = _dispatch(lib, ids, w, h, E, noalloc=False)
        got = _dispatch(lib, ids, w, h, E, noalloc=True)
        for r, x in zip(ref, got):
            assert torch.equal(r, x), f'call {call}'
        assert int(got[0][-1]) == T * k


def test_noalloc_dispatch_rejects_oversize_call():
    lib = _lib.load()
    T, k, E = 256 * 513, 1, 64            # ceil(T/256) * E = 32832 > 32768 entries
    dev = torch.device('cuda', 0)
    ids = torch.zeros((T, k), dtype=torch.int32, device=dev)
    w = torch.zeros((T, k), dtype=torch.float32, device=dev)
    bufs = [torch.empty(n, dtype=t, device=dev) for n, t in
            ((E + 1, torch.int32), (T * k, torch.int32), (T * k, torch.int32), (T * k, torch.float32))]
    st = lib.b200q_moe_dispatch_noalloc_dev(ids.data_ptr(), w.data_ptr(), T, k, E, None, 0,
                                            *[b.data_ptr() for b in bufs], None,
                                            torch.cuda.current_stream().cuda_stream)
    assert st == _lib.B200Q_EINVAL
    assert b'static scratch limit' in lib.b200q_last_error()


def test_noalloc_dispatch_reports_bad_expert_id():
    """A bad expert id through the allocation-free entry point is reported by
    b200q_check_device_error (the error word lives in the static array) and
    the call otherwise equals the regular dispatch."""
    lib = _lib.load()
    torch.cuda.set_device(0)
    assert lib.b200q_check_device_error() == 0
    T, k, E, D = 300, 2, 8, 128
    g = torch.Generator(device='cuda')
    g.manual_seed(11)
    ids = torch.topk(torch.rand((T, E), generator=g, device='cuda'), k, dim=1).indices.to(torch.int32)
    ids[17, 1] = E + 3
    ids = ids.contiguous()
    w = torch.rand((T, k), generator=g, device='cuda')
    h = torch.randn((T, D), generator=g, device='cuda')
    ref = _dispatch(lib, ids, w, h, E, noalloc=False)
    assert lib.b200q_check_device_error() == 2
    got = _dispatch(lib, ids, w, h, E, noalloc=True)
    assert lib.b200q_check_device_error() == 2
    assert lib.b200q_check_device_error() == 0
    n = T * k - 1
    assert int(got[0][-1]) == n and int(got[1][17 * k + 1]) == -1
    for i, (r, x) in enumerate(zip(ref, got)):
        if i in (2, 3, 4):                   # token_of, slot_w, xperm: the unassigned tail is not written
            r, x = r[:n], x[:n]
        assert torch.equal(r, x)
