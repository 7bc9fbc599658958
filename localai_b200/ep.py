"""Expert parallelism for the quantised MoE layer across the GPUs of one node.

The reference runs the MoE block on one CPU process (engine/zaya.py:274-307).
Here the experts are sharded over G ranks (one process per GPU, NCCL over
NVLink/NVSwitch) and the T tokens are sharded evenly; per layer call:

    1. every rank routes its own tokens (router + softmax top-k);
    2. the (token, j) pairs are sorted by (owner rank, local expert) with the
       stable counting sort, rows gathered as bf16;
    3. all-to-all of the per-(rank, expert) row counts, then all-to-all of the
       rows (variable splits);
    4. the received rows, ordered (source rank, local expert), run in place
       through the grouped tensor-core GEMMs (gate/up with fused SiLU*up,
       then down, bf16 rows), one GEMM group per (source, expert) run;
    5. all-to-all of the expert outputs (bf16) back to the source ranks;
    6. weighted combine in fixed j order.

Expert placement is greedy LPT on expected per-expert loads with E/G experts
per rank, which keeps the busiest rank close to the mean under a skewed
(Zipf) router.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .moe import QuantMoE


def lpt_placement(loads, n_ranks):
    """Greedy longest-processing-time placement with E/G experts per rank.

    Returns (owner[E], local_index[E]); experts of a rank are numbered in
    ascending global index.
    """
    loads = np.asarray(loads, dtype=np.float64)
    E = loads.size
    if E % n_ranks:
        raise ValueError('expert count must be divisible by the number of ranks')
    cap = E // n_ranks
    owner = np.empty(E, np.int64)
    rank_load = np.zeros(n_ranks)
    rank_n = np.zeros(n_ranks, np.int64)
    for e in np.argsort(-loads, kind='stable'):
        free = np.nonzero(rank_n < cap)[0]
        r = free[np.argmin(rank_load[free])]
        owner[e] = r
        rank_load[r] += loads[e]
        rank_n[r] += 1
    local = np.empty(E, np.int64)
    for r in range(n_ranks):
        mine = np.nonzero(owner == r)[0]
        local[mine] = np.arange(mine.size)
    return owner, local


class EPMoE:
    """One rank's share of an expert-parallel QuantMoE.

    ``layer`` holds the full router and this rank's experts (``gate_up``/
    ``down`` of its E/G local experts, in local-index order; built with
    ``local_experts=E/G``).
    """

    def __init__(self, layer: QuantMoE, owner, local, group=None):
        self.layer = layer
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = layer.E
        self.E_loc = self.E // self.G
        owner = np.asarray(owner)
        local = np.asarray(local)
        dev = layer.router_w.device
        # virtual expert index: experts ordered by (owner rank, local index)
        self.virt = torch.from_numpy((owner * self.E_loc + local).astype(np.int32)).to(dev)
        # GEMM group (source rank, local expert) -> local expert
        self.group_w = torch.arange(self.E_loc, dtype=torch.int32, device=dev).repeat(self.G)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        L = self.layer
        T, dev = h.shape[0], h.device
        h = h.contiguous()
        _, ids, w = L.route(h)
        vids = self.virt[ids.long()]
        offsets, slot_of, _, slot_w, xsend = L.dispatch(h, vids, w)
        cnt_send = (offsets[1:] - offsets[:-1]).view(self.G, self.E_loc).contiguous()
        cnt_recv = torch.empty_like(cnt_send)
        dist.all_to_all_single(cnt_recv, cnt_send, group=self.group)
        counts = torch.stack([cnt_send.sum(1), cnt_recv.sum(1)]).cpu()      # one host sync per call
        send_splits, recv_splits = counts[0].tolist(), counts[1].tolist()
        R = int(sum(recv_splits))
        xrecv = torch.empty((R, L.D), dtype=xsend.dtype, device=dev)
        dist.all_to_all_single(xrecv, xsend, recv_splits, send_splits, group=self.group)
        # Received rows are ordered (source rank, local expert); each such run is
        # one GEMM group whose weights are its local expert -- no regrouping copy.
        grp_off = torch.zeros(self.G * self.E_loc + 1, dtype=torch.int32, device=dev)
        grp_off[1:] = torch.cumsum(cnt_recv.reshape(-1), 0).to(torch.int32)
        if R > 0:
            out_recv = L.experts(xrecv, grp_off, None, group_w=self.group_w)
        else:
            out_recv = torch.empty((0, L.D), dtype=torch.bfloat16, device=dev)
        back = torch.empty((xsend.shape[0], L.D), dtype=out_recv.dtype, device=dev)
        dist.all_to_all_single(back, out_recv, send_splits, recv_splits, group=self.group)
        return L.combine(back, slot_of, T, slot_w)

    __call__ = forward
