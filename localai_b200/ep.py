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

Two transports carry steps 3-5:

* ``'nccl'``: NCCL ``all_to_all_single`` (counts, then rows with variable
  splits, which needs one host synchronisation for the split sizes, then the
  outputs); received rows form one GEMM group per (source rank, local expert).
* ``'p2p'``: device-initiated exchange over NVLink peer memory (CUDA IPC
  mappings of every rank's exchange region, plain stores, epoch flags; no
  host synchronisation): a count-exchange kernel builds the layouts, a send
  kernel gathers each routed row as bf16 straight into its owner's receive
  buffer (expert-major, so each local expert is one GEMM group), and the down
  GEMM's epilogue stores each output row straight into its source rank's
  return buffer.  Needs peer access between all ranks' GPUs.  The call's
  epoch lives on the device, so with ``graph=True`` (default) a layer call is
  captured once per token count in a CUDA graph and replayed (no per-call
  host work between the kernels).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .moe import QuantMoE, _stream, pipelined_host_forward


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

    def __init__(self, layer: QuantMoE, owner, local, group=None, *, transport: str = 'nccl',
                 max_tokens: int | None = None, graph: bool = True, fused: bool = True):
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
        if transport not in ('nccl', 'p2p'):
            raise ValueError("transport must be 'nccl' or 'p2p'")
        if transport == 'p2p' and layer.t_dn != layer.type:
            # the device-side exchange entries run both expert GEMMs with one weight type
            raise NotImplementedError("transport 'p2p' needs gate/up and down experts of one GGML type")
        self.transport = transport
        self.ctx = None
        self.use_graph = graph
        # library kernels launched by graph replays (the library's own launch
        # counter sees only the capture)
        self.graph_launches = 0
        # p2p: the row exchange runs inside the gate/up GEMM (push warps, per-expert
        # arrival flags); False: a separate send kernel, then the GEMMs
        self.fused = fused
        self._graphs = {}
        if transport == 'p2p':
            if max_tokens is None or max_tokens < 1:
                raise ValueError('the p2p transport needs max_tokens (tokens per rank per call)')
            self._open_p2p(int(max_tokens), dev)

    # -- p2p transport --------------------------------------------------------
    def _open_p2p(self, max_tokens: int, dev):
        L, lib = self.layer, self.layer.lib
        self.max_tokens = max_tokens
        cap_send = max_tokens * L.k
        cap_recv = self.G * cap_send
        ctx = ctypes.c_void_p()
        _lib.check(lib.b200q_ep_create(self.G, self.rank, self.E_loc, L.D, cap_send, cap_recv, ctypes.byref(ctx)))
        self.ctx = ctx
        nb = int(lib.b200q_ep_handle_bytes())
        mine = (ctypes.c_uint8 * nb)()
        _lib.check(lib.b200q_ep_handle(ctx, mine))
        t = torch.tensor(list(bytes(mine)), dtype=torch.uint8, device=dev)
        every = torch.empty(self.G * nb, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(every, t, group=self.group)
        handles = bytes(every.cpu().numpy().tobytes())
        _lib.check(lib.b200q_ep_open(ctx, handles))
        dist.barrier(group=self.group)
        self.act = torch.empty((cap_recv, L.F), dtype=torch.bfloat16, device=dev)

    def close(self):
        """Release the p2p exchange region (collective: every rank calls it)."""
        if self.ctx is not None:
            torch.cuda.synchronize()
            self._graphs.clear()
            dist.barrier(group=self.group)
            _lib.check(self.layer.lib.b200q_ep_destroy(self.ctx))
            self.ctx = None

    def _forward_p2p(self, h: torch.Tensor, marks: list | None = None) -> torch.Tensor:
        L, lib = self.layer, self.layer.lib
        T, dev = h.shape[0], h.device
        if T > self.max_tokens:
            raise ValueError(f'{T} tokens exceed max_tokens={self.max_tokens}')

        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))

        ep = 0                      # device-side epoch: advanced by the count exchange
        mark('start')
        hb = torch.empty((T, L.D), dtype=torch.bfloat16, device=dev)
        _, ids, w = L.route(h, hb)
        mark('route')
        vids = self.virt[ids.long()]
        offsets, slot_of, token_of, slot_w, _ = L.dispatch(h, vids, w, gather=False)
        mark('dispatch')
        st = _stream()
        _lib.check(lib.b200q_ep_exchange_counts_dev(self.ctx, offsets.data_ptr(), ep, st))
        mark('counts')
        if self.fused:
            # rows stored into the owners' buffers by the gate/up GEMM's own push warps
            _lib.check(lib.b200q_ep_dispatch_experts_dev(
                self.ctx, L.type, L.gate_up.data_ptr(), L.gu_stride, L.down.data_ptr(), L.dn_stride, L.F,
                self.act.data_ptr(), hb.data_ptr(), T, token_of.data_ptr(), offsets.data_ptr(), T * L.k, ep, 0, st))
            mark('send+experts')
        else:
            _lib.check(lib.b200q_ep_send_rows_bf16_dev(self.ctx, hb.data_ptr(), T, token_of.data_ptr(),
                                                       offsets.data_ptr(), T * L.k, ep, st))
            mark('send')
            _lib.check(lib.b200q_ep_experts_dev(self.ctx, L.type, L.gate_up.data_ptr(), L.gu_stride,
                                                L.down.data_ptr(), L.dn_stride, L.F, self.act.data_ptr(), ep, 0, st))
            mark('experts')
        y = torch.empty((T, L.D), dtype=torch.float32, device=dev)
        _lib.check(lib.b200q_ep_combine_dev(self.ctx, slot_of.data_ptr(), slot_w.data_ptr(), T, L.k, y.data_ptr(),
                                            ep, st))
        mark('combine')
        return y

    def phase_times(self, h: torch.Tensor) -> dict:
        """One p2p layer call with CUDA events between its stages; returns the
        milliseconds of each stage on this rank ('experts' includes the wait
        for every rank's rows, 'combine' the wait for the returned outputs).
        Collective: every rank calls it."""
        if self.transport != 'p2p':
            raise ValueError('phase_times needs the p2p transport')
        marks = []
        self._forward_p2p(h.contiguous(), marks)
        torch.cuda.synchronize()
        out = {marks[i][0]: round(marks[i - 1][1].elapsed_time(marks[i][1]), 4) for i in range(1, len(marks))}
        out['total'] = round(marks[0][1].elapsed_time(marks[-1][1]), 4)
        return out

    def forward_host(self, h_host: torch.Tensor, y_host: torch.Tensor | None = None, chunks: int = 4):
        """forward() on this rank's host (pinned) tokens with the PCIe copies
        overlapped with the computation; every rank must use the same number
        of chunks."""
        return pipelined_host_forward(self.forward, h_host, y_host, chunks, self.layer.router_w.device)

    def _forward_graph(self, h: torch.Tensor) -> torch.Tensor:
        """p2p layer call through a CUDA graph captured on the first call for
        this token count (every rank captures at the same call)."""
        T = h.shape[0]
        entry = self._graphs.get(T)
        if entry is None:
            static_h = torch.empty_like(h)
            side = torch.cuda.Stream(h.device)
            side.wait_stream(torch.cuda.current_stream(h.device))
            with torch.cuda.stream(side):
                static_h.copy_(h)
                self._forward_p2p(static_h)          # eager call: allocations settle (all ranks alike)
            torch.cuda.current_stream(h.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            n0 = self.layer.lib.b200q_launch_count()
            with torch.cuda.graph(graph):
                y_static = self._forward_p2p(static_h)
            n_kernels = self.layer.lib.b200q_launch_count() - n0      # library kernels in the graph
            entry = (graph, static_h, y_static, n_kernels)
            self._graphs[T] = entry
        graph, static_h, y_static, n_kernels = entry
        static_h.copy_(h)
        graph.replay()
        self.graph_launches += n_kernels
        return y_static.clone()

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        if self.transport == 'p2p':
            if self.use_graph:
                return self._forward_graph(h.contiguous())
            return self._forward_p2p(h.contiguous())
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
