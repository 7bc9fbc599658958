"""Quantised mixture-of-experts FFN on the GPU.

The reference block (engine/zaya.py:274-307, ``ZayaModel._moe``) routes one
token at a time to one expert and runs two GEMVs on it.  ``QuantMoE`` runs the
same block batched over T tokens and generalised to top-k:

    logits = h @ Wr^T (+ router bias), hb = bf16(h)   b200q_moe_route_bf16_dev
    p = softmax(logits); top-k of p (+ sel bias)      (same call)
    stable counting sort of (token, j) by expert      b200q_moe_dispatch_dev
    xperm[slot_of[t, j]] = hb[t]                      b200q_moe_scatter_bf16_dev
    act = SiLU(gate x) * (up x)  per expert           b200q_gemm_dev (gate/up mode, tcgen05)
    out = w_slot * (down act)    per expert           b200q_gemm_dev (plain mode, tcgen05; bf16 rows)
    y[t] = sum_j out[slot(t, j)]                      b200q_moe_combine_dev

Expert weights are raw GGUF Q4_K, Q5_K, Q6_K, Q8_0 or Q4_0 tensors in ZAYA's layout:
``gate_up`` [E, 2F, D] (gate rows first, then up rows, as
``np.split(packed, 2)`` reads them, engine/zaya.py:304) and ``down``
[E, D, F_pad] with F_pad the next multiple of the type's block (256 for the
K-quants, 32 for Q8_0; padded values decode to zero).  Rows whose byte size
is not a multiple of 16 (e.g. Q6_K with 1024 columns, 840 B) are copied once
into 16-byte-padded rows, which the tensor-core GEMM loads with TMA.
"""
from __future__ import annotations

import torch

from . import _lib
from .ops import packed_row_bytes, pad_rows

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 8, 12, 13, 14


def _stream():
    return torch.cuda.current_stream().cuda_stream


def chunk_bounds(T: int, chunks: int) -> list[int]:
    """Token boundaries of the chunks of pipelined_host_forward.  The first
    chunk's upload and the last chunk's download overlap nothing, so with
    three or more chunks those two are half the size of the others; no chunk
    is empty."""
    chunks = max(1, min(chunks, T))
    wts = [1.0] * chunks
    if chunks >= 3:
        wts[0] = wts[-1] = 0.5
    acc = [0.0]
    for wv in wts:
        acc.append(acc[-1] + wv)
    return sorted({int(round(T * a / acc[-1])) for a in acc})


def pipelined_host_forward(fn, h_host: torch.Tensor, y_host: torch.Tensor | None, chunks: int, device):
    """y_host = fn(h) for host (pinned) f32 h_host [T, D], in ``chunks`` token
    chunks: the host->device copy of chunk c+1 and the device->host copy of
    chunk c-1 run on their own streams while ``fn`` computes chunk c on the
    current stream.  Returns y_host after the last copy has been queued; the
    copies are ordered before any later work on the current stream."""
    if h_host.is_cuda or h_host.dtype != torch.float32 or h_host.dim() != 2:
        raise ValueError('h_host must be a host f32 [T, D] tensor')
    T, D = h_host.shape
    if y_host is None:
        y_host = torch.empty((T, D), dtype=torch.float32, pin_memory=True)
    bounds = chunk_bounds(T, chunks)
    chunks = len(bounds) - 1
    rows = max(bounds[c + 1] - bounds[c] for c in range(chunks))
    comp = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    s_in.wait_stream(comp)          # buffers below may reuse memory the current stream just released
    s_out.wait_stream(comp)
    hbuf = [torch.empty((rows, D), dtype=torch.float32, device=device) for _ in range(min(2, chunks))]
    freed = [None, None]            # event: compute has finished reading hbuf[i]
    done_out = []
    for c in range(chunks):
        a, b = bounds[c], bounds[c + 1]
        buf = hbuf[c % 2][: b - a]
        with torch.cuda.stream(s_in):
            if freed[c % 2] is not None:
                s_in.wait_event(freed[c % 2])
            buf.copy_(h_host[a:b], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(s_in)
        comp.wait_event(ready)
        y = fn(buf)
        ev = torch.cuda.Event()
        ev.record(comp)
        freed[c % 2] = ev
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev)
            y_host[a:b].copy_(y, non_blocking=True)
            y.record_stream(s_out)
            fin = torch.cuda.Event()
            fin.record(s_out)
            done_out.append(fin)
    for b in hbuf:
        b.record_stream(s_in)
    comp.wait_event(done_out[-1])
    return y_host


class QuantMoE:
    def __init__(self, router_w: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor, *, d_model: int,
                 d_ff: int, top_k: int, router_bias: torch.Tensor | None = None,
                 sel_bias: torch.Tensor | None = None, renormalize: bool = True, ggml_type: int = Q4_K,
                 local_experts: int | None = None, down_type: int | None = None):
        down_type = ggml_type if down_type is None else down_type
        for t in (ggml_type, down_type):
            if t not in (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K):
                raise NotImplementedError('the tensor-core expert path supports Q4_0, Q8_0, Q4_K, Q5_K and Q6_K '
                                          'expert weights')
        if d_ff % 64 or d_model % 128 or (ggml_type not in (Q4_0, Q8_0) and d_model % 256):
            raise ValueError('d_ff must be a multiple of 64 and d_model of 128 (256 for K-quant gate/up)')
        self.E = router_w.shape[0]
        self.D, self.F, self.k = d_model, d_ff, top_k
        # GGML types of the gate/up and the down experts (mixed quantisations
        # may keep the down projection at higher precision)
        self.type, self.t_dn = ggml_type, down_type
        blk = 32 if down_type in (Q4_0, Q8_0) else 256
        self.F_pad = (d_ff + blk - 1) // blk * blk
        self.router_w = router_w.contiguous().float()
        self.router_bias = None if router_bias is None else router_bias.contiguous().float()
        self.sel_bias = None if sel_bias is None else sel_bias.contiguous().float()
        self.renorm = 1 if renormalize else 0
        self.gate_up = gate_up.contiguous()
        self.down = down.contiguous()
        # expert tensors may hold a subset of the experts (expert parallelism)
        self.E_held = self.E if local_experts is None else local_experts
        rb_gu, rb_dn = packed_row_bytes(ggml_type, d_model), packed_row_bytes(down_type, self.F_pad)
        gu_bytes = self.E_held * 2 * d_ff * rb_gu
        dn_bytes = self.E_held * d_model * rb_dn
        if self.gate_up.numel() != gu_bytes or self.down.numel() != dn_bytes:
            raise ValueError(f'expert tensors must be {gu_bytes} and {dn_bytes} bytes of GGML types {ggml_type} '
                             f'and {down_type}')
        # device copies with 16-byte rows where the packed rows are not
        self.gate_up, self.gu_stride = pad_rows(self.gate_up, self.E_held * 2 * d_ff, rb_gu)
        self.down, self.dn_stride = pad_rows(self.down, self.E_held * d_model, rb_dn)
        self.lib = _lib.load()
        # decode-sized batches (T * k slots up to this) take the grouped GEMV path
        self.small_slots = min(self.lib.b200q_gemv_grouped_max_tokens(ggml_type, d_model),
                               self.lib.b200q_gemv_grouped_max_tokens(down_type, self.F_pad))

    # -- stages ---------------------------------------------------------------
    def route(self, h: torch.Tensor, hb: torch.Tensor | None = None):
        """Router logits, top-k expert ids and routing weights; with ``hb``
        (bf16 [T, D]) also hb = bf16(h)."""
        T = h.shape[0]
        dev = h.device
        logits = torch.empty((T, self.E), dtype=torch.float32, device=dev)
        ids = torch.empty((T, self.k), dtype=torch.int32, device=dev)
        w = torch.empty((T, self.k), dtype=torch.float32, device=dev)
        nws = self.lib.b200q_moe_route_workspace_bytes(T, self.E, self.D)
        ws = torch.empty(nws // 4, dtype=torch.float32, device=dev) if nws else None
        args = (h.data_ptr(), self.router_w.data_ptr(),
                None if self.router_bias is None else self.router_bias.data_ptr(),
                None if self.sel_bias is None else self.sel_bias.data_ptr(),
                T, self.E, self.D, self.k, self.renorm, logits.data_ptr(), ids.data_ptr(), w.data_ptr(),
                None if ws is None else ws.data_ptr(), nws)
        if hb is None:
            _lib.check(self.lib.b200q_moe_route_dev(*args, _stream()))
        else:
            if hb.dtype != torch.bfloat16 or hb.shape != (T, self.D) or not hb.is_contiguous():
                raise ValueError('hb must be a contiguous bf16 [T, d_model] tensor')
            _lib.check(self.lib.b200q_moe_route_bf16_dev(*args, hb.data_ptr(), _stream()))
        return logits, ids, w

    def topk(self, logits: torch.Tensor):
        T = logits.shape[0]
        ids = torch.empty((T, self.k), dtype=torch.int32, device=logits.device)
        w = torch.empty((T, self.k), dtype=torch.float32, device=logits.device)
        _lib.check(self.lib.b200q_moe_topk_dev(
            logits.data_ptr(), None if self.sel_bias is None else self.sel_bias.data_ptr(),
            T, self.E, self.k, self.renorm, ids.data_ptr(), w.data_ptr(), _stream()))
        return ids, w

    def dispatch(self, h: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, gather: bool = True,
                 n_experts: int | None = None, k: int | None = None):
        """Stable counting sort of the (token, j) pairs by expert id; rows
        gathered as bf16 when ``gather``.  ``n_experts``/``k`` override the
        layer's (ZAYA routes over experts + 1 with k = 1)."""
        E = self.E if n_experts is None else n_experts
        k = self.k if k is None else k
        T, dev = ids.shape[0], ids.device
        S = T * k
        nblk = self.lib.b200q_moe_num_blocks(T)
        scratch = torch.empty((2, nblk * E), dtype=torch.int32, device=dev)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        slot_of = torch.empty(S, dtype=torch.int32, device=dev)
        token_of = torch.empty(S, dtype=torch.int32, device=dev)
        slot_w = torch.empty(S, dtype=torch.float32, device=dev)
        xperm = torch.empty((S, self.D), dtype=torch.bfloat16, device=dev) if gather else None
        _lib.check(self.lib.b200q_moe_dispatch_dev(
            ids.data_ptr(), w.data_ptr(), T, k, E, h.data_ptr() if gather else None, self.D,
            scratch[0].data_ptr(), scratch[1].data_ptr(), offsets.data_ptr(), slot_of.data_ptr(),
            token_of.data_ptr(), slot_w.data_ptr(), None if xperm is None else xperm.data_ptr(), _stream()))
        return offsets, slot_of, token_of, slot_w, xperm

    def scatter_bf16(self, hb: torch.Tensor, slot_of: torch.Tensor, S: int) -> torch.Tensor:
        """xperm[slot_of[t, j]] = hb[t]: the rows of gather_bf16, each token row
        read once and stored k times."""
        xperm = torch.empty((S, self.D), dtype=torch.bfloat16, device=hb.device)
        _lib.check(self.lib.b200q_moe_scatter_bf16_dev(hb.data_ptr(), hb.shape[0], slot_of.data_ptr(), self.k, S,
                                                       self.D, xperm.data_ptr(), _stream()))
        return xperm

    def gather_bf16(self, hb: torch.Tensor, token_of: torch.Tensor) -> torch.Tensor:
        """xperm[s] = hb[token_of[s]] (bf16 rows grouped by expert)."""
        S = token_of.numel()
        xperm = torch.empty((S, self.D), dtype=torch.bfloat16, device=hb.device)
        _lib.check(self.lib.b200q_moe_gather_bf16_dev(hb.data_ptr(), hb.shape[0], token_of.data_ptr(), S, self.D,
                                                      xperm.data_ptr(), _stream()))
        return xperm

    def experts(self, xperm: torch.Tensor, offsets: torch.Tensor, slot_w: torch.Tensor | None, *,
                group_w: torch.Tensor | None = None, out_dtype=torch.bfloat16, max_ctas: int = 0):
        """Grouped gate/up (fused SiLU*up) then grouped down, on the tensor cores.

        ``slot_w`` scales each output row (None: unscaled).  With ``group_w``
        the rows form ``len(group_w)`` groups whose experts are
        ``group_w[g]`` among the experts this layer holds (expert parallelism
        feeds the rows received from every rank this way, in place)."""
        S, dev = xperm.shape[0], xperm.device
        groups = offsets.numel() - 1
        gw = None if group_w is None else group_w.data_ptr()
        act = torch.empty((S, self.F), dtype=torch.bfloat16, device=dev)
        _lib.check(self.lib.b200q_gemm_dev(
            self.type, xperm.data_ptr(), S, self.D, self.gate_up.data_ptr(), self.gu_stride, groups, 2 * self.F,
            self.F, self.F, offsets.data_ptr(), gw, self.E_held, None, 0, 0, None, act.data_ptr(), self.F,
            max_ctas, _stream()))
        out = torch.empty((S, self.D), dtype=out_dtype, device=dev)
        _lib.check(self.lib.b200q_gemm_dev(
            self.t_dn, act.data_ptr(), S, self.F, self.down.data_ptr(), self.dn_stride, groups, self.D, -1, self.D,
            offsets.data_ptr(), gw, self.E_held, out.data_ptr(), 1 if out_dtype == torch.bfloat16 else 0, self.D,
            None if slot_w is None else slot_w.data_ptr(), None, 0, max_ctas, _stream()))
        return out

    def combine(self, out: torch.Tensor, slot_of: torch.Tensor, T: int, slot_w: torch.Tensor | None = None,
                k: int | None = None):
        """y[t] = sum_j (slot_w) * out[slot(t, j)]; pass slot_w when out is unweighted."""
        y = torch.empty((T, self.D), dtype=torch.float32, device=out.device)
        _lib.check(self.lib.b200q_moe_combine_dev(out.data_ptr(), 1 if out.dtype == torch.bfloat16 else 0,
                                                  slot_of.data_ptr(), None if slot_w is None else slot_w.data_ptr(),
                                                  T, self.k if k is None else k, self.D, y.data_ptr(), _stream()))
        return y

    def experts_small(self, h: torch.Tensor, offsets: torch.Tensor, token_of: torch.Tensor, *,
                      n_groups: int | None = None):
        """Decode path: f32 rows of the routed tokens through grouped GEMVs
        (gate/up, silu*up, down) with f32 accumulation; returns unweighted
        f32 [slots, D].  Experts without tokens read no weights."""
        S, dev = token_of.numel(), h.device
        G = self.E_held if n_groups is None else n_groups
        xs = torch.empty((S, self.D), dtype=torch.float32, device=dev)
        _lib.check(self.lib.b200q_moe_gather_f32_dev(h.data_ptr(), h.shape[0], token_of.data_ptr(), S, self.D,
                                                     xs.data_ptr(), _stream()))
        gu = torch.empty((S, 2 * self.F), dtype=torch.float32, device=dev)
        active = max(1, min(G, S))
        _lib.check(self.lib.b200q_gemv_grouped_dev(
            self.type, self.gate_up.data_ptr(), 2 * self.F * self.gu_stride, self.gu_stride, G, offsets.data_ptr(),
            xs.data_ptr(), gu.data_ptr(), 2 * self.F, 2 * self.F, self.D, S, S, active, _stream()))
        if self.F_pad != self.F:
            act = torch.zeros((S, self.F_pad), dtype=torch.float32, device=dev)
        else:
            act = torch.empty((S, self.F_pad), dtype=torch.float32, device=dev)
        _lib.check(self.lib.b200q_silu_mul_dev(gu.data_ptr(), S, self.F, act.data_ptr(), self.F_pad, _stream()))
        out = torch.empty((S, self.D), dtype=torch.float32, device=dev)
        _lib.check(self.lib.b200q_gemv_grouped_dev(
            self.t_dn, self.down.data_ptr(), self.D * self.dn_stride, self.dn_stride, G, offsets.data_ptr(),
            act.data_ptr(), out.data_ptr(), self.D, self.D, self.F_pad, S, S, active, _stream()))
        return out

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """y[T, D] for hidden states h[T, D] (f32).  Up to ``small_slots``
        routed rows take the grouped-GEMV decode path (f32 accumulation),
        larger batches the tensor-core path (bf16 operands)."""
        if h.dtype != torch.float32 or not h.is_cuda or h.dim() != 2 or h.shape[1] != self.D:
            raise ValueError('h must be a CUDA f32 [T, d_model] tensor')
        h = h.contiguous()
        T = h.shape[0]
        if T * self.k <= self.small_slots:
            _, ids, w = self.route(h)
            offsets, slot_of, token_of, slot_w, _ = self.dispatch(h, ids, w, gather=False)
            out = self.experts_small(h, offsets, token_of)
            return self.combine(out, slot_of, T, slot_w)
        hb = torch.empty((T, self.D), dtype=torch.bfloat16, device=h.device)
        _, ids, w = self.route(h, hb)
        offsets, slot_of, token_of, slot_w, _ = self.dispatch(h, ids, w, gather=False)
        xperm = (self.scatter_bf16(hb, slot_of, token_of.numel()) if self.k <= 32
                 else self.gather_bf16(hb, token_of))
        out = self.experts(xperm, offsets, slot_w)
        return self.combine(out, slot_of, T)

    def forward_host(self, h_host: torch.Tensor, y_host: torch.Tensor | None = None, chunks: int = 4,
                     device=None) -> torch.Tensor:
        """forward() on host (pinned) hidden states, overlapping the PCIe copies
        with the layer computation chunk by chunk (see pipelined_host_forward)."""
        device = device or self.router_w.device
        return pipelined_host_forward(self.forward, h_host, y_host, chunks, device)

    __call__ = forward
