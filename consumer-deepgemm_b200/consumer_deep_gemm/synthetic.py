"""Seeded synthetic MoE GEMM workloads (the shapes and distributions of the benchmark configs).

No public dataset or checkpoint is involved: activations are N(0,1) BF16 rows,
weights N(0, 0.02), quantised with ``per_block_cast_to_fp8`` (1x128 FP32 scales)
and ``per_block_cast_to_fp4`` (MXFP4, UE8M0 per 32).  Routed rows are laid out
the way vLLM's ``deepgemm_moe_permute`` does it: experts in increasing order,
each expert's rows first, its region padded to a multiple of 128 rows whose
``m_indices`` entry is -1.

Configs (``CONFIGS``):
  c0  E=8,   K=512,  N=256,  1024 rows, per-expert counts from a seeded multinomial
  c1  E=256, K=4096, N=4096, 64 tokens x top-8 uniform (decode FC1)
  c2  E=256, K=2048, N=4096, 8192 tokens x top-8 uniform, A = silu(g)*u (prefill FC2)
  c3  E=256, K=4096, N=4096, 16384 tokens x top-8, Zipf(1.2) expert popularity
  c4  the expert-parallel layer: 32768 tokens x top-8, FC1 K=N=4096, FC2 K=2048, N=4096
  c2u, c3u  c2 and c3 with UE8M0 activation scales: each 1x128 scale rounded up to a
      power of two and the block requantised with it (the DeepGEMM UE8M0 recipe for
      SM100 activations); not a benchmark config of the reference, a second data format
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from deep_gemm.utils.math import per_block_cast_to_fp4, per_block_cast_to_fp8

ALIGN = 128


@dataclass(frozen=True)
class Config:
    name: str
    num_experts: int
    k: int
    n: int
    tokens: int
    topk: int
    routing: str  # "uniform" | "zipf" | "multinomial"
    swiglu_input: bool = False
    ue8m0_scales: bool = False  # activation scales rounded up to powers of two


CONFIGS = {
    "c0": Config("c0", 8, 512, 256, 1024, 1, "multinomial"),
    "c1": Config("c1", 256, 4096, 4096, 64, 8, "uniform"),
    "c2": Config("c2", 256, 2048, 4096, 8192, 8, "uniform", swiglu_input=True),
    "c3": Config("c3", 256, 4096, 4096, 16384, 8, "zipf"),
    "c2u": Config("c2u", 256, 2048, 4096, 8192, 8, "uniform", swiglu_input=True, ue8m0_scales=True),
    "c3u": Config("c3u", 256, 4096, 4096, 16384, 8, "zipf", ue8m0_scales=True),
    "c4_fc1": Config("c4_fc1", 256, 4096, 4096, 32768, 8, "uniform"),
    "c4_fc2": Config("c4_fc2", 256, 2048, 4096, 32768, 8, "uniform", swiglu_input=True),
}


def route(cfg: Config, seed: int = 0) -> torch.Tensor:
    """Expert ids ``[tokens, topk]`` (int64, CPU) for a config's routing law."""
    g = torch.Generator().manual_seed(seed)
    e = cfg.num_experts
    if cfg.routing == "multinomial":
        ids = torch.multinomial(torch.ones(e), cfg.tokens * cfg.topk, replacement=True, generator=g)
        return ids.view(cfg.tokens, cfg.topk)
    if cfg.routing == "uniform":
        return torch.rand(cfg.tokens, e, generator=g).topk(cfg.topk, dim=1).indices
    if cfg.routing == "zipf":
        perm = torch.randperm(e, generator=g)
        logp = -1.2 * torch.log(torch.arange(1, e + 1, dtype=torch.float64))
        gumbel = -torch.log(-torch.log(torch.rand(cfg.tokens, e, generator=g, dtype=torch.float64)))
        ranks = (logp.unsqueeze(0) + gumbel).topk(cfg.topk, dim=1).indices
        return perm[ranks]
    raise ValueError(cfg.routing)


def contiguous_layout(topk_ids: torch.Tensor, num_experts: int, align: int = ALIGN):
    """Expert-major, ``align``-padded layout of routed rows.

    Returns ``(m_indices int32 [M_pad], src_token int64 [M_pad])`` where
    ``src_token`` is the token each row copies (-1 on padding rows).
    """
    flat = topk_ids.reshape(-1).to(torch.int64)
    tok = torch.arange(topk_ids.shape[0]).repeat_interleave(topk_ids.shape[1])
    counts = torch.bincount(flat, minlength=num_experts)
    padded = (counts + align - 1) // align * align
    starts = torch.cumsum(padded, 0) - padded
    m_pad = int(padded.sum())
    m_indices = torch.full((m_pad,), -1, dtype=torch.int32)
    src = torch.full((m_pad,), -1, dtype=torch.int64)
    order = torch.argsort(flat, stable=True)
    sorted_e = flat[order]
    first = torch.cumsum(counts, 0) - counts
    pos = starts[sorted_e] + (torch.arange(flat.numel()) - first[sorted_e])
    m_indices[pos] = sorted_e.to(torch.int32)
    src[pos] = tok[order]
    return m_indices, src


def make_inputs(cfg: Config, device="cpu", seed: int = 0, weight_device=None):
    """Quantised operands of one config.

    Returns a dict with ``a`` (fp8 [M_pad, K]), ``sa`` (fp32 [M_pad, K/128]),
    ``b`` (uint8 [E, N, K/2]), ``sb`` (uint8 [E, N, K/32]), ``m_indices``
    (int32 [M_pad]) and the bookkeeping ``rows`` (routed rows R), ``m_pad``.
    Padding rows carry zeros with scale 1.  Routing and activations come from a
    CPU generator, weights from a generator on ``weight_device`` (default
    ``device``), so the same seed gives the same routing everywhere.
    """
    weight_device = weight_device or device
    ids = route(cfg, seed)
    m_indices, src = contiguous_layout(ids, cfg.num_experts)
    g = torch.Generator().manual_seed(seed + 1)
    if cfg.swiglu_input:
        gate = torch.randn(cfg.tokens, cfg.k, generator=g, dtype=torch.float32).to(torch.bfloat16)
        up = torch.randn(cfg.tokens, cfg.k, generator=g, dtype=torch.float32).to(torch.bfloat16)
        x = (torch.nn.functional.silu(gate.float()) * up.float()).to(torch.bfloat16)
    else:
        x = torch.randn(cfg.tokens, cfg.k, generator=g, dtype=torch.float32).to(torch.bfloat16)
    xq, xs = per_block_cast_to_fp8(x.to(device).float())
    if cfg.ue8m0_scales:
        xs = torch.exp2(torch.ceil(torch.log2(xs)))
        xb = x.to(device).float().view(cfg.tokens, cfg.k // 128, 128) / xs.unsqueeze(-1)
        xq = xb.view(cfg.tokens, cfg.k).to(torch.float8_e4m3fn)
    valid = src >= 0
    m_pad = m_indices.numel()
    a = torch.zeros(m_pad, cfg.k, dtype=torch.float8_e4m3fn, device=device)
    sa = torch.ones(m_pad, cfg.k // 128, dtype=torch.float32, device=device)
    vidx = valid.nonzero().flatten().to(device)
    a[vidx] = xq[src[valid].to(device)]
    sa[vidx] = xs[src[valid].to(device)]
    b, sb = make_weights(cfg.num_experts, cfg.n, cfg.k, weight_device, seed + 2)
    return {
        "a": a, "sa": sa, "b": b.to(device), "sb": sb.to(device),
        "m_indices": m_indices.to(device), "rows": int(valid.sum()), "m_pad": m_pad,
        "src_token": src, "cfg": cfg,
    }


def make_weights(num_experts: int, n: int, k: int, device="cpu", seed: int = 2, chunk: int = 8):
    """MXFP4 expert weights ``W ~ N(0, 0.02)`` quantised expert by expert."""
    g = torch.Generator(device=device).manual_seed(seed)
    b = torch.empty(num_experts, n, k // 2, dtype=torch.uint8, device=device)
    sb = torch.empty(num_experts, n, k // 32, dtype=torch.uint8, device=device)
    for e0 in range(0, num_experts, chunk):
        e1 = min(num_experts, e0 + chunk)
        w = torch.randn(e1 - e0, n, k, generator=g, device=device, dtype=torch.float32) * 0.02
        b[e0:e1], sb[e0:e1] = per_block_cast_to_fp4(w)
    return b, sb
