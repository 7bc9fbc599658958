"""Worker for tests/test_ep_gpu.py: one process per GPU (launched by torchrun).

Every rank builds the same small MoE layer, runs its token shard through the
expert-parallel layer (its E/G experts, NCCL all-to-all) and through a full
single-GPU QuantMoE, and exits non-zero if they differ.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from localai_b200 import synth                       # noqa: E402
from localai_b200.ep import EPMoE, lpt_placement     # noqa: E402
from localai_b200.moe import QuantMoE                # noqa: E402


def main():
    rank, world = int(os.environ['RANK']), int(os.environ['WORLD_SIZE'])
    dev = torch.device('cuda', int(os.environ['LOCAL_RANK']))
    torch.cuda.set_device(dev)
    dist.init_process_group('nccl', timeout=timedelta(seconds=120), device_id=dev)
    E, D, F, k, T = 16, 512, 128, 4, 1024
    rng = np.random.default_rng(0)
    gate_up = [synth.q4_k(rng, 2 * F, D) for _ in range(E)]
    down = [synth.q4_k(rng, D, 256, zero_tail_cols=256 - F) for _ in range(E)]
    wr = torch.from_numpy(rng.normal(0, D ** -0.5, size=(E, D)).astype(np.float32)).to(dev)
    bias = torch.from_numpy(np.log(np.arange(1, E + 1) ** -1.1).astype(np.float32)).to(dev)
    h = torch.from_numpy(rng.normal(size=(T, D)).astype(np.float32)).to(dev)
    cat = lambda parts: torch.frombuffer(bytearray(b''.join(parts)), dtype=torch.uint8).to(dev)
    full = QuantMoE(wr, cat(gate_up), cat(down), d_model=D, d_ff=F, top_k=k, router_bias=bias)
    _, ids, _ = full.route(h)
    loads = torch.bincount(ids.reshape(-1).long(), minlength=E).cpu().numpy()
    owner, local = lpt_placement(loads, world)
    mine = [int(e) for e in np.nonzero(owner == rank)[0]]
    part = QuantMoE(wr, cat([gate_up[e] for e in mine]), cat([down[e] for e in mine]), d_model=D, d_ff=F,
                    top_k=k, router_bias=bias, local_experts=len(mine))
    ep = EPMoE(part, owner, local)
    n = T // world
    shard = h[rank * n:(rank + 1) * n]
    y_ep = ep(shard)
    # single-GPU reference with the same arithmetic as the expert-parallel
    # path (unweighted bf16 expert rows, routing weight applied in the combine):
    # every GEMM row is independent of how rows are grouped, so the two must
    # agree bit for bit
    _, ids_s, w_s = full.route(shard)
    off, slot_of, _, slot_w, xperm = full.dispatch(shard, ids_s, w_s)
    y_same = full.combine(full.experts(xperm, off, None), slot_of, n, slot_w)
    y_fwd = full(shard)
    torch.cuda.synchronize()
    err = float((y_ep - y_same).abs().max() / y_same.abs().max())
    err_fwd = float((y_ep - y_fwd).abs().max() / y_fwd.abs().max())
    good = err == 0.0 and err_fwd < 1e-2
    print(f'rank {rank}: ep vs single-GPU (same rounding) {err:.3e}, vs forward {err_fwd:.3e}', flush=True)
    # peer-memory transport: same arithmetic, so bit-identical to the NCCL path;
    # several calls in a row (epochs), one of them with a ragged shard
    p2p = EPMoE(part, owner, local, transport='p2p', max_tokens=n)
    for it in range(3):
        y_p = p2p(shard)
        d = float((y_p - y_ep).abs().max())
        print(f'rank {rank}: p2p call {it} vs nccl max |diff| {d:.3e}', flush=True)
        good = good and d == 0.0
    # the captured graph reads new inputs (same token count, other values)
    other = shard.flip(0).contiguous()
    d = float((p2p(other) - ep(other)).abs().max())
    print(f'rank {rank}: p2p replay on new inputs vs nccl max |diff| {d:.3e}', flush=True)
    good = good and d == 0.0
    # the eager (non-graph) p2p paths alternate with the graph replays: rows
    # stored by the gate/up GEMM's push warps (fused), or by a separate send
    # kernel before the GEMMs
    for fused in (True, False):
        p2p_eager = EPMoE(part, owner, local, transport='p2p', max_tokens=n, graph=False, fused=fused)
        for it in range(2):
            d = float((p2p_eager(shard) - y_ep).abs().max())
            print(f'rank {rank}: p2p eager (fused={fused}) call {it} vs nccl max |diff| {d:.3e}', flush=True)
            good = good and d == 0.0
        p2p_eager.close()
    m = n - 3 - rank                        # ragged: a different token count on every rank
    y_p = p2p(shard[:m])
    y_n = ep(shard[:m])
    d = float((y_p - y_n).abs().max())
    print(f'rank {rank}: p2p ragged ({m} tokens) vs nccl max |diff| {d:.3e}', flush=True)
    good = good and d == 0.0
    torch.cuda.synchronize()
    st = full.lib.b200q_check_device_error()
    good = good and st == 0
    p2p.close()
    ok = torch.tensor([1 if good else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if int(ok.item()) == 1 else 1)


if __name__ == '__main__':
    main()
