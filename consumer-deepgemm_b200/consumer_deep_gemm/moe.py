"""Mixture-of-experts layer on the grouped FP8 x MXFP4 GEMM, with expert parallelism.

``MoELayer.forward(x, topk_ids, topk_w)`` computes, for every token t::

    y[t] = sum_j topk_w[t, j] * FC2_e( act( FC1_e( q(x[t]) ) ) ),   e = topk_ids[t, j]

with q = 1x128 e4m3 quantisation (per_block_cast_to_fp8 semantics), FC1/FC2 the
grouped GEMM of this package (MXFP4 weights, gate = first half of FC1's output),
and act = 1x128 e4m3 quantisation of silu(gate) * up.  This is the sequence vLLM's
DeepGemmFP4Experts runs around ``m_grouped_fp8_fp4_gemm_nt_contiguous``
(vllm/model_executor/layers/fused_moe/experts/deep_gemm_moe.py:485-545).

One rank: the forward has no host synchronisation (group offsets computed on the device,
layout sized for the worst case), so it can be captured in a CUDA graph.

Expert parallelism: with a process group of N ranks, rank r owns experts
[r*E/N, (r+1)*E/N).  Each rank quantises its own tokens, exchanges per-expert row
counts (one small all-to-all and the only host synchronisation), sends every
routed row to the rank owning its expert (one all-to-all of packed rows: e4m3
data, FP32 scales and the local expert id in one byte row of
``native row_bytes(H)``), lays the received rows out per local expert with 128-row
alignment, runs FC1 -> act -> FC2, and sends the rows back (all-to-all of BF16
rows) for the weighted top-k sum.  Collectives go through torch.distributed
(NCCL on GPUs); all compute runs in libcdg_b200.so kernels.

With ``max_tokens_per_rank`` set, the exchange needs no host synchronisation: every
rank quantises and packs its rows straight into a fixed-capacity region per
destination (``max_tokens_per_rank * topk`` rows after a header row holding the
per-expert counts), one equal-split all-to-all moves rows and counts together, the
receiver derives the group layout from the headers on the device, and the GEMMs run
over the worst-case padded row count, leaving rows outside every group unwritten.
All ranks must use the same value and pass at most that many tokens.

``exchange="p2p"`` (with ``max_tokens_per_rank``, GPUs of one NVLink domain) replaces
the collectives by the library's own peer-memory exchange: each rank owns an exchange
window shared through CUDA IPC; the dispatch kernel quantises each token's row once and
stores it straight into the window of every rank that owns one of its experts (one row per
token and rank, listing the token's local experts there), the receiver expands it into the
experts' groups, FC2's epilogue stores each of its rows straight back into the source's
window at the row's slot (a row table the receiver's permute writes; ``fused_return=False``
uses a separate return kernel instead), and release/acquire flags (bounded waits) order the
steps.

The device steps sit behind a small ``ops`` interface so that the exchange
logic can also be exercised with CPU implementations (tests do that with the
gloo backend).
"""

from __future__ import annotations

import numpy as np
import torch

from . import native
from .gemm import m_grouped_fp8_fp4_gemm_nt_contiguous
from .layout import transform_sf_into_required_layout

ALIGN = 128


def _output(m, n, device, d_rows):
    """The GEMM's BF16 [m, n] output, or, when a row table routes the rows elsewhere, a
    [1, n] placeholder expanded to [m, n] that only gives the shape."""
    if d_rows is None:
        return torch.empty(m, n, dtype=torch.bfloat16, device=device)
    return torch.empty(1, n, dtype=torch.bfloat16, device=device).expand(m, n)


class NativeOps:
    """Device kernels of libcdg_b200.so through the torch binding."""

    # the quantising steps can write the GEMM's activation planes directly (FP32 1x128 recipe)
    supports_planes = True

    def __init__(self):
        self.C = native.require()

    def quant_dispatch_local_planes(self, x, topk_ids, num_experts, expert_off, m_pad):
        return self.C.ep_quant_dispatch_local_planes(x, topk_ids, num_experts, expert_off, m_pad)

    def act_planes(self, h, m_indices):
        return self.C.silu_mul_quant_planes(h, m_indices)

    def gemm_planes(self, planes, row_exp, w, w_sf, m_indices, skip_ungrouped=False, d_rows=None):
        d = _output(planes.shape[1], w.shape[1], planes.device, d_rows)
        self.C.grouped_gemm_planes(planes, row_exp, w, w_sf, d, m_indices, 4 if skip_ungrouped else 0, d_rows)
        return None if d_rows is not None else d

    def quant(self, x, ue8m0=False):
        return self.C.quant_fp8_rows(x, ue8m0)

    def count(self, topk_ids, num_experts):
        return self.C.ep_count(topk_ids, num_experts)

    def count_offsets(self, topk_ids, num_experts):
        return self.C.ep_count_offsets(topk_ids, num_experts)

    def pack(self, xq, xs, topk_ids, num_experts, ranks, send_off, rows):
        return self.C.ep_pack(xq, xs, topk_ids, num_experts, ranks, send_off, rows)

    def permute(self, rows, hidden, local_experts, expert_off, m_pad):
        return self.C.ep_permute(rows, hidden, local_experts, expert_off, m_pad)

    def quant_pack_fixed(self, x, topk_ids, num_experts, ranks, cap, ue8m0=False):
        return self.C.ep_quant_pack_fixed(x, topk_ids, num_experts, ranks, cap, ue8m0)

    def quant_dispatch_local(self, x, topk_ids, num_experts, expert_off, m_pad, ue8m0=False):
        return self.C.ep_quant_dispatch_local(x, topk_ids, num_experts, expert_off, m_pad, ue8m0)

    def permute_fixed(self, rows, hidden, local_experts, ranks, cap, m_pad):
        return self.C.ep_permute_fixed(rows, hidden, local_experts, ranks, cap, m_pad)

    def gemm(self, a, sa, w, w_sf, m_indices, skip_ungrouped=False, d_rows=None):
        d = _output(a.shape[0], w.shape[1], a.device, d_rows)
        m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (w, w_sf), d, m_indices, _skip_ungrouped_rows=skip_ungrouped,
                                             _d_rows=d_rows)
        return None if d_rows is not None else d

    def act(self, h, m_indices, ue8m0=False):
        return self.C.silu_mul_quant(h, m_indices, ue8m0)

    def unpermute(self, y, perm_pos):
        return self.C.ep_unpermute(y, perm_pos)

    def combine(self, rows, send_index, topk_w):
        return self.C.ep_combine(rows, send_index, topk_w)

    def unpermute_combine(self, y, perm_pos, send_index, topk_w):
        return self.C.ep_unpermute_combine(y, perm_pos, send_index, topk_w)


def _all_to_all(out, inp, out_splits, in_splits, group):
    import torch.distributed as dist

    dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)
    return out


class PeerWindows:
    """The exchange windows of all ranks of `group`, mapped into this process (CUDA IPC)."""

    def __init__(self, group, max_tokens: int, topk: int, hidden: int, device):
        import torch.distributed as dist

        self.C = native.require()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.topk = max_tokens, topk
        nbytes = self.C.ep_window_bytes(self.world, max_tokens, topk, hidden)
        if nbytes == 0:
            raise ValueError("unsupported peer exchange shape")
        self.own, handle = self.C.ep_window_create(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        ptrs, self.opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.own)
            else:
                ptrs.append(self.C.ep_window_open(h))
                self.opened.append(ptrs[-1])
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)  # every window is mapped everywhere before the first store

    def status(self) -> int:
        """0, or a nonzero code when a bounded wait on another rank's flag gave up."""
        return self.C.ep_window_status(self.own)

    def close(self):
        for p in self.opened:
            self.C.ep_window_close(p, True)
        self.opened = []
        if self.own:
            self.C.ep_window_close(self.own, False)
            self.own = 0


class MoELayer:
    """An MoE layer whose experts are sharded over the ranks of ``group``.

    w1: packed e2m1 [E_local, 2*I, H/2] (gate rows first), w1_scale UE8M0 [E_local, 2*I, H/32];
    w2: packed e2m1 [E_local, H, I/2], w2_scale UE8M0 [E_local, H, I/32].
    ``num_experts`` is the global E; E_local = E / world size.  With ``w2=None`` the layer
    is the expert-parallel grouped GEMM alone: y[t] = sum_j topk_w[t, j] * FC1_e(q(x[t])).
    ``ue8m0=True`` quantises the activations (q and act) with power-of-two scales, the UE8M0
    recipe DeepGEMM's SM100 path uses (1x128 scale amax/448 rounded up to a power of two,
    kept as FP32); the GEMMs then run their direct class (one MMA per K slice).
    """

    def __init__(self, w1, w1_scale, w2=None, w2_scale=None, num_experts: int = 0, group=None, ops=None,
                 max_tokens_per_rank: int | None = None, exchange: str = "nccl", ue8m0: bool = False,
                 planes: bool | None = None, fused_return: bool = True):
        self.ops = ops or NativeOps()
        self.ue8m0 = bool(ue8m0)
        # FP32 activation scales: the quantising steps write the GEMMs' activation planes directly
        # (the GEMMs then skip their own plane split); power-of-two scales need no planes
        self.planes = (not self.ue8m0 and getattr(self.ops, "supports_planes", False)) if planes is None else \
            bool(planes) and not self.ue8m0
        self.max_tokens = max_tokens_per_rank
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        if exchange == "p2p" and max_tokens_per_rank is None:
            raise ValueError("the peer-memory exchange needs max_tokens_per_rank (fixed capacity)")
        self.exchange = exchange
        # peer exchange: FC2's epilogue stores each row straight into its source's window
        # (the GEMM's row table) instead of a separate return kernel
        self.fused_return = bool(fused_return)
        self.windows = None
        self.group = group
        if group is not None:
            import torch.distributed as dist

            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if num_experts % self.world:
            raise ValueError("the number of experts must divide evenly over the ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        if w1.shape[0] != self.local_experts or (w2 is not None and w2.shape[0] != self.local_experts):
            raise ValueError("w1/w2 must hold this rank's experts")
        # weight scale layout prepared once (the weight-load hook)
        self.w1 = w1.view(torch.uint8)
        self.w1_sf = transform_sf_into_required_layout(w1_scale) if w1.is_cuda else w1_scale
        self.w2 = w2.view(torch.uint8) if w2 is not None else None
        if w2 is not None:
            self.w2_sf = transform_sf_into_required_layout(w2_scale) if w2.is_cuda else w2_scale
        self.out_dim = w2.shape[1] if w2 is not None else w1.shape[1]
        self.inter = w1.shape[1] // 2
        # optional callable(name), called after each step of a forward has been launched
        # (dispatch, permute, fc1, act, fc2, return, combine; no return with the fused return):
        # a profiler records CUDA events
        # there to split the step's device time by phase
        self.on_phase = None

    def _phase(self, name):
        if self.on_phase is not None:
            self.on_phase(name)

    def status(self) -> int:
        """0, CDG_ERR_DEVICE_INDEX (9) when a kernel skipped an access it could not make, or
        CDG_ERR_DEVICE_TIMEOUT (6) when one of this process's device waits gave up
        since the last call: a wait on another rank's exchange flag (this layer's window) or a
        GEMM pipeline wait.  Synchronises the device and clears the library's record."""
        st = self.windows.status() if self.windows is not None else 0
        dev, _ = native.read_device_status(True)
        return st or dev

    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor) -> torch.Tensor:
        if self.world > 1 and self.exchange == "p2p":
            return self._forward_p2p(x, topk_ids, topk_w)
        if self.world > 1 and self.max_tokens is not None:
            return self._forward_fixed(x, topk_ids, topk_w)
        ops, world, E, E_loc = self.ops, self.world, self.num_experts, self.local_experts
        dev = x.device
        topk_ids = topk_ids.contiguous()
        topk_w = topk_w.to(torch.float32).contiguous()
        if world == 1:
            return self._forward_local(x, topk_ids, topk_w)
        # split-size exchange
        xq, xs = ops.quant(x, self.ue8m0)
        counts = ops.count(topk_ids, E)                                  # [E] rows per global expert
        both = torch.empty(2, E, dtype=counts.dtype, device=dev)
        both[0] = counts
        _all_to_all(both[1], counts, None, None, self.group)
        # the one host synchronisation of the layer (one copy): split sizes and the local layout
        mats = both.cpu().numpy().astype(np.int64).reshape(2, world, E_loc)
        send_splits = mats[0].sum(1)
        recv_splits = mats[1].sum(1)
        aligned = (mats[1].sum(0) + ALIGN - 1) // ALIGN * ALIGN
        m_pad = int(aligned.sum())
        offs = np.concatenate([np.cumsum(aligned) - aligned, np.cumsum(send_splits) - send_splits])
        offs = torch.from_numpy(offs).to(dev, non_blocking=False)
        expert_off, send_off = offs[:E_loc], offs[E_loc:]
        send_splits, recv_splits = send_splits.tolist(), recv_splits.tolist()

        sent, send_index = ops.pack(xq, xs, topk_ids, E, world, send_off, sum(send_splits))
        recv = _all_to_all(torch.empty(sum(recv_splits), sent.shape[1], dtype=sent.dtype, device=dev), sent,
                           recv_splits, send_splits, self.group)

        if m_pad > 0:
            a, sa, m_indices, perm_pos = ops.permute(recv, x.shape[1], E_loc, expert_off, m_pad)
            h = ops.gemm(a, sa, self.w1, self.w1_sf, m_indices)
            if self.w2 is not None:
                aq, asc = ops.act(h, m_indices, self.ue8m0)
                h = ops.gemm(aq, asc, self.w2, self.w2_sf, m_indices)
            back = ops.unpermute(h, perm_pos)
        else:
            back = torch.empty(0, self.out_dim, dtype=torch.bfloat16, device=dev)
        out_rows = _all_to_all(torch.empty(sent.shape[0], self.out_dim, dtype=back.dtype, device=dev), back,
                               send_splits, recv_splits, self.group)
        return ops.combine(out_rows, send_index, topk_w)

    def _forward_local(self, x, topk_ids, topk_w):
        """One rank, no exchange, no host synchronisation: the group offsets are computed on the
        device and the layout is sized for the worst case (every group 127 rows short of a
        multiple of 128); each token's row is quantised once straight into it, and the combine
        reads the GEMM's rows through the permutation."""
        ops, E = self.ops, self.num_experts
        T, topk = topk_ids.shape
        if hasattr(ops, "count_offsets"):
            _, expert_off = ops.count_offsets(topk_ids, E)               # group starts, on the device
        else:
            counts = ops.count(topk_ids, E)                              # [E] rows per expert
            aligned = (counts.to(torch.int64) + ALIGN - 1) // ALIGN * ALIGN
            expert_off = torch.cumsum(aligned, 0) - aligned
        m_pad = (T * topk + (ALIGN - 1) * E + ALIGN - 1) // ALIGN * ALIGN
        if self.planes:
            pl, rexp, m_indices, perm_pos, send_index = ops.quant_dispatch_local_planes(x, topk_ids, E, expert_off,
                                                                                        m_pad)
            self._phase("dispatch")
            h = ops.gemm_planes(pl, rexp, self.w1, self.w1_sf, m_indices, skip_ungrouped=True)
        else:
            a, sa, m_indices, perm_pos, send_index = ops.quant_dispatch_local(x, topk_ids, E, expert_off, m_pad,
                                                                              self.ue8m0)
            self._phase("dispatch")
            h = ops.gemm(a, sa, self.w1, self.w1_sf, m_indices, skip_ungrouped=True)
        self._phase("fc1")
        if self.w2 is not None:
            h = self._act_fc2(h, m_indices)
        y = ops.unpermute_combine(h, perm_pos, send_index, topk_w)
        self._phase("combine")
        return y

    def _act_fc2(self, h, m_indices, d_rows=None):
        """SiLU-mul + requant of FC1's rows, then FC2 (rows outside every group left unwritten;
        with ``d_rows``, row r is stored at address d_rows[r] and nothing is returned)."""
        ops = self.ops
        route = {} if d_rows is None else {"d_rows": d_rows}
        if self.planes:
            pl, rexp = ops.act_planes(h, m_indices)
            self._phase("act")
            out = ops.gemm_planes(pl, rexp, self.w2, self.w2_sf, m_indices, skip_ungrouped=True, **route)
        else:
            aq, asc = ops.act(h, m_indices, self.ue8m0)
            self._phase("act")
            out = ops.gemm(aq, asc, self.w2, self.w2_sf, m_indices, skip_ungrouped=True, **route)
        self._phase("fc2")
        return out

    def _forward_fixed(self, x, topk_ids, topk_w):
        """Exchange without a host synchronisation: fixed per-destination capacity."""
        ops, world, E, E_loc, group = self.ops, self.world, self.num_experts, self.local_experts, self.group
        dev = x.device
        T, topk = topk_ids.shape
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens_per_rank={self.max_tokens}")
        cap = self.max_tokens * topk  # rows any one destination can receive from this rank
        topk_ids = topk_ids.contiguous()
        topk_w = topk_w.to(torch.float32).contiguous()
        sent, send_index = ops.quant_pack_fixed(x, topk_ids, E, world, cap, self.ue8m0)
        recv = _all_to_all(torch.empty_like(sent), sent, None, None, group)
        m_pad = (world * cap + 127 * E_loc + ALIGN - 1) // ALIGN * ALIGN
        a, sa, m_indices, perm_pos = ops.permute_fixed(recv, x.shape[1], E_loc, world, cap, m_pad)
        h = ops.gemm(a, sa, self.w1, self.w1_sf, m_indices, skip_ungrouped=True)
        if self.w2 is not None:
            aq, asc = ops.act(h, m_indices, self.ue8m0)
            h = ops.gemm(aq, asc, self.w2, self.w2_sf, m_indices, skip_ungrouped=True)
        back = ops.unpermute(h, perm_pos)
        out_rows = _all_to_all(torch.empty_like(back), back, None, None, group)
        return ops.combine(out_rows, send_index, topk_w)

    def _forward_p2p(self, x, topk_ids, topk_w):
        """Fixed capacity, rows moved by the library's own peer-memory stores (no collective)."""
        C, world, E, E_loc = native.require(), self.world, self.num_experts, self.local_experts
        T, topk = topk_ids.shape
        H = x.shape[1]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens_per_rank={self.max_tokens}")
        if self.out_dim != H:
            raise ValueError("the peer-memory exchange returns rows of the input width")
        cap = self.max_tokens * topk
        if self.windows is None:
            self.windows = PeerWindows(self.group, self.max_tokens, topk, H, x.device)
        win, me = self.windows, self.rank
        if win.topk != topk:
            raise ValueError(f"the exchange windows were made for top-{win.topk} routing, got top-{topk}")
        send_index = C.ep_dispatch_p2p(x, topk_ids.contiguous(), E, world, self.max_tokens, win.peers, win.own, me,
                                       self.ue8m0)
        self._phase("dispatch")
        m_pad = (world * cap + 127 * E_loc + ALIGN - 1) // ALIGN * ALIGN
        # fused return: the permute also writes FC2's row table (each row's place in its source's
        # window), FC2 stores there, and the combine raises this rank's return flags
        fused = self.fused_return and self.w2 is not None
        table_peers = win.peers if fused else None
        if self.planes:
            pl, rexp, m_indices, ret_slot, ret_rows = C.ep_permute_p2p_planes(
                win.own, world, self.max_tokens, topk, H, E_loc, m_pad, x, table_peers)
            self._phase("permute")
            h = self.ops.gemm_planes(pl, rexp, self.w1, self.w1_sf, m_indices, skip_ungrouped=True)
        else:
            a, sa, m_indices, ret_slot, ret_rows = C.ep_permute_p2p(win.own, world, self.max_tokens, topk, H, E_loc,
                                                                    m_pad, x, table_peers)
            self._phase("permute")
            h = self.ops.gemm(a, sa, self.w1, self.w1_sf, m_indices, skip_ungrouped=True)
        self._phase("fc1")
        if fused:
            self._act_fc2(h, m_indices, d_rows=ret_rows)
        else:
            if self.w2 is not None:
                h = self._act_fc2(h, m_indices)
            C.ep_return_p2p(h, ret_slot, world, self.max_tokens, topk, win.peers, win.own, me)
            self._phase("return")
        y = C.ep_combine_p2p(win.own, send_index, topk_w.to(torch.float32).contiguous(), world, self.max_tokens, H,
                             table_peers, me)
        self._phase("combine")
        return y

    def capture(self, x, topk_ids, topk_w):
        """Record one forward on these (static) input tensors in a CUDA graph.

        Returns (graph, output): ``graph.replay()`` reruns the forward on whatever the input
        tensors then hold and writes the result into ``output``.  Needs the peer-memory
        exchange (every step of it reads its step number on the device) or a single rank
        (whose forward has no host synchronisation).
        The first forward (window set-up, library initialisation) runs here, outside the graph.
        """
        if self.world > 1 and self.exchange != "p2p":
            raise ValueError("graph capture needs exchange='p2p' (the collectives' split sizes are host values)")
        self.forward(x, topk_ids, topk_w)  # set-up outside the graph
        torch.cuda.synchronize(x.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = self.forward(x, topk_ids, topk_w)
        return g, out

    def close(self):
        """Release the peer exchange windows (all ranks, after their last forward)."""
        if self.windows is not None:
            self.windows.close()
            self.windows = None

    __call__ = forward
