"""CPU reference of the MoE layer steps (test infrastructure).

``TorchRefOps`` implements the ``ops`` interface of consumer_deep_gemm.moe.MoELayer
on CPU tensors with plain torch and the oracle GEMM, in a fixed row order.  With
it, ``MoELayer`` over world size 1 is the reference layer, and over a gloo
process group it exercises the expert-parallel exchange logic without a GPU.
"""

import torch

from deep_gemm.utils.math import per_block_cast_to_fp8
from oracle import cdg_oracle as oracle


def row_bytes(hidden):
    """Bytes of one dispatched row: e4m3 data, FP32 scale per 128 columns, int32 expert id, padded to 16."""
    return (hidden + 4 * (hidden // 128) + 4 + 15) // 16 * 16


def cast_to_fp8_pow2(x):
    """1x128 e4m3 quantisation with power-of-two scales (the UE8M0 recipe of DeepGEMM's SM100
    path): s = amax / 448 (amax clamped at 1e-12) rounded up to a power of two, q = e4m3(x / s)."""
    m, k = x.shape
    xv = x.float().view(m, k // 128, 128)
    s = xv.abs().amax(dim=2).clamp(min=1e-12) / 448.0
    mant, ex = torch.frexp(s)  # s = mant * 2^ex, mant in [0.5, 1): a power of two iff mant == 0.5
    s2 = torch.where(mant == 0.5, s, torch.ldexp(torch.ones_like(s), ex))
    return (xv / s2.unsqueeze(-1)).to(torch.float8_e4m3fn).view(m, k), s2


class TorchRefOps:
    def quant(self, x, ue8m0=False):
        return cast_to_fp8_pow2(x) if ue8m0 else per_block_cast_to_fp8(x.float())

    def count(self, topk_ids, num_experts):
        ids = topk_ids.flatten().long()
        ids = ids[(ids >= 0) & (ids < num_experts)]
        return torch.bincount(ids, minlength=num_experts).to(torch.int32)

    def pack(self, xq, xs, topk_ids, num_experts, ranks, send_off, rows):
        """Packed rows [rows, row_bytes(H)] uint8: e4m3 data | FP32 scales | int32 local expert."""
        T, k = topk_ids.shape
        H = xq.shape[1]
        per_rank = num_experts // ranks
        out = torch.zeros(rows, row_bytes(H), dtype=torch.uint8)
        send_index = torch.full((T * k,), -1, dtype=torch.int32)
        fill = [0] * ranks
        for i, e in enumerate(topk_ids.flatten().tolist()):
            if not 0 <= e < num_experts:
                continue
            d = e // per_rank
            r = int(send_off[d]) + fill[d]
            fill[d] += 1
            out[r, :H] = xq[i // k].view(torch.uint8)
            out[r, H:H + 4 * (H // 128)] = xs[i // k].contiguous().view(torch.uint8)
            out[r, H + 4 * (H // 128):H + 4 * (H // 128) + 4] = torch.tensor([e % per_rank], dtype=torch.int32).view(
                torch.uint8)
            send_index[i] = r
        return out, send_index

    def permute(self, rows, hidden, local_experts, expert_off, m_pad):
        H, nkb = hidden, hidden // 128
        a = torch.zeros(m_pad, H, dtype=torch.float8_e4m3fn)
        sa = torch.ones(m_pad, nkb, dtype=torch.float32)
        m_indices = torch.full((m_pad,), -1, dtype=torch.int32)
        pos = torch.empty(rows.shape[0], dtype=torch.int32)
        fill = [0] * local_experts
        for i in range(rows.shape[0]):
            e = int(rows[i, H + 4 * nkb:H + 4 * nkb + 4].contiguous().view(torch.int32)[0])
            p = int(expert_off[e]) + fill[e]
            fill[e] += 1
            a[p] = rows[i, :H].contiguous().view(torch.float8_e4m3fn)
            sa[p] = rows[i, H:H + 4 * nkb].contiguous().view(torch.float32)
            m_indices[p], pos[i] = e, p
        return a, sa, m_indices, pos

    def quant_pack_fixed(self, x, topk_ids, num_experts, ranks, cap, ue8m0=False):
        """Regions of 1 + cap packed rows per destination: header (int32 counts per local expert), rows."""
        T, k = topk_ids.shape
        H = x.shape[1]
        per_rank = num_experts // ranks
        xq, xs = self.quant(x, ue8m0)
        out = torch.zeros(ranks * (cap + 1), row_bytes(H), dtype=torch.uint8)
        send_index = torch.full((T * k,), -1, dtype=torch.int32)
        fill = [0] * ranks
        cnt = torch.zeros(ranks, per_rank, dtype=torch.int32)
        for i, e in enumerate(topk_ids.flatten().tolist()):
            if not 0 <= e < num_experts:
                continue
            d = e // per_rank
            slot = fill[d]
            fill[d] += 1
            cnt[d, e % per_rank] += 1
            if slot >= cap:
                continue
            r = d * (cap + 1) + 1 + slot
            out[r, :H] = xq[i // k].view(torch.uint8)
            out[r, H:H + 4 * (H // 128)] = xs[i // k].contiguous().view(torch.uint8)
            out[r, H + 4 * (H // 128):H + 4 * (H // 128) + 4] = torch.tensor([e % per_rank], dtype=torch.int32).view(
                torch.uint8)
            send_index[i] = r
        for d in range(ranks):
            out[d * (cap + 1), :4 * per_rank] = cnt[d].view(torch.uint8)
        return out, send_index

    def quant_dispatch_local(self, x, topk_ids, num_experts, expert_off, m_pad, ue8m0=False):
        """One rank: quantised rows straight into the contiguous layout, slots in order."""
        T, k = topk_ids.shape
        H = x.shape[1]
        xq, xs = self.quant(x, ue8m0)
        a = torch.zeros(m_pad, H, dtype=torch.float8_e4m3fn)
        sa = torch.ones(m_pad, H // 128, dtype=torch.float32)
        m_indices = torch.full((m_pad,), -1, dtype=torch.int32)
        perm_pos = torch.full((T * k,), -1, dtype=torch.int32)
        send_index = torch.full((T * k,), -1, dtype=torch.int32)
        fill = [0] * num_experts
        for i, e in enumerate(topk_ids.flatten().tolist()):
            if not 0 <= e < num_experts:
                continue
            p = int(expert_off[e]) + fill[e]
            fill[e] += 1
            a[p], sa[p], m_indices[p] = xq[i // k], xs[i // k], e
            perm_pos[i], send_index[i] = p, i
        return a, sa, m_indices, perm_pos, send_index

    def permute_fixed(self, rows, hidden, local_experts, ranks, cap, m_pad):
        """Fixed-capacity receive buffer: source r's header at row r*(cap+1), its rows after it."""
        H, nkb = hidden, hidden // 128
        counts = torch.stack([rows[r * (cap + 1), :4 * local_experts].contiguous().view(torch.int32)
                              for r in range(ranks)])
        tot = counts.long().sum(0)
        aligned = (tot + 127) // 128 * 128
        off = torch.cumsum(aligned, 0) - aligned
        a = torch.zeros(m_pad, H, dtype=torch.float8_e4m3fn)
        sa = torch.ones(m_pad, nkb, dtype=torch.float32)
        m_indices = torch.full((m_pad,), -1, dtype=torch.int32)
        pos = torch.full((rows.shape[0],), -1, dtype=torch.int32)
        fill = [0] * local_experts
        for r in range(ranks):
            for slot in range(int(counts[r].sum())):
                i = r * (cap + 1) + 1 + slot
                e = int(rows[i, H + 4 * nkb:H + 4 * nkb + 4].contiguous().view(torch.int32)[0])
                p = int(off[e]) + fill[e]
                fill[e] += 1
                a[p] = rows[i, :H].contiguous().view(torch.float8_e4m3fn)
                sa[p] = rows[i, H:H + 4 * nkb].contiguous().view(torch.float32)
                m_indices[p], pos[i] = e, p
        return a, sa, m_indices, pos

    def gemm(self, a, sa, w, w_sf, m_indices, skip_ungrouped=False):
        d = torch.empty(a.shape[0], w.shape[1], dtype=torch.bfloat16)
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (w, w_sf), d, m_indices)
        return d

    def act(self, h, m_indices, ue8m0=False):
        i = h.shape[1] // 2
        g, u = h[:, :i].float(), h[:, i:].float()
        v = torch.nn.functional.silu(g) * u
        return cast_to_fp8_pow2(v) if ue8m0 else per_block_cast_to_fp8(v)

    def unpermute(self, y, perm_pos):
        out = torch.zeros(perm_pos.numel(), y.shape[1], dtype=y.dtype)
        ok = perm_pos >= 0
        out[ok] = y[perm_pos[ok].long()]
        return out

    def unpermute_combine(self, y, perm_pos, send_index, topk_w):
        return self.combine(self.unpermute(y, perm_pos), send_index, topk_w)

    def combine(self, rows, send_index, topk_w):
        T, k = topk_w.shape
        y = torch.zeros(T, rows.shape[1], dtype=torch.float32)
        for i, r in enumerate(send_index.tolist()):
            if r >= 0:
                y[i // k] += topk_w[i // k, i % k] * rows[r].float()
        return y.to(torch.bfloat16)


def make_layer_inputs(tokens, experts, hidden, inter, topk, seed=0):
    """Seeded tokens, routing and MXFP4 expert weights for a small layer."""
    from deep_gemm.utils.math import per_block_cast_to_fp4

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16)
    ids = torch.rand(tokens, experts, generator=g).topk(topk, dim=1).indices.to(torch.int32)
    w = torch.rand(tokens, topk, generator=g)
    w = w / w.sum(1, keepdim=True)
    w1, w1s = per_block_cast_to_fp4(torch.randn(experts, 2 * inter, hidden, generator=g) * 0.05)
    w2, w2s = per_block_cast_to_fp4(torch.randn(experts, hidden, inter, generator=g) * 0.05)
    return x, ids, w, w1, w1s, w2, w2s
