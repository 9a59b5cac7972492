"""CPU oracle for the grouped FP8 x MXFP4 MoE GEMM (TEST INFRASTRUCTURE ONLY).

This module is a checker, never a product path.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The CUDA library never calls into it and the
Python package never falls back to it.

It restates, on CPU tensors, the reference's Python dequant + matmul path of
lmxxf/Consumer-DeepGEMM (``consumer_deep_gemm/gemm.py``), function by function,
with the same roundings:

* activations are dequantised in BF16: ``bf16(bf16(fp8) * bf16(scale))``
  (gemm.py:31-52), a BF16/FP32 ``a`` passes through and ignores its scale
  (gemm.py:33-34);
* weights are decoded from packed E2M1 (low nibble = even k) through the OCP
  table and multiplied by ``2**(e-127)`` (UE8M0) or by a float scale in FP32,
  then rounded to BF16 (gemm.py:147-187, gemm.py:16-28, gemm.py:55-59);
* ``d`` is zeroed, then every group is an FP32 ``torch.mm`` whose result is cast
  to ``d.dtype`` and scattered with ``index_copy_`` (gemm.py:343-367), groups
  visited in increasing id so that, for overlapping psum ranges, the last group
  wins exactly as in the reference;
* ``m_indices`` is either one id per row or a vector of cumulative group ends
  (psum form) when its length equals the number of groups but not M
  (gemm.py:303-329).  Ids outside ``[0, G)`` select no group, so those rows stay 0.

Parity is pinned against the reference itself: ``tests/golden/make_golden.py``
imports the reference in the build container and stores its outputs as
fixtures, and ``tests/test_oracle_golden.py`` checks this module against them
bit for bit.
"""

from __future__ import annotations

import numpy as np
import torch

# OCP MX E2M1 code points (gemm.py:16-28).
E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def dequant_fp8_block(x: torch.Tensor, scale: torch.Tensor, block_k: int = 128) -> torch.Tensor:
    """BF16 activation dequant; follows gemm.py:31-52 step for step."""
    if x.dtype in (torch.bfloat16, torch.float32):
        return x
    m, k = x.shape[0], x.shape[1]
    if scale.dim() == 2 and scale.shape[1] > 1:
        block_k = k // scale.shape[1]
    n_blocks = (k + block_k - 1) // block_k
    pad = n_blocks * block_k - k
    if pad:
        x = torch.nn.functional.pad(x.view(torch.uint8), (0, pad)).view(x.dtype)
    xf = x.reshape(m, n_blocks, block_k).to(torch.bfloat16)
    s = scale.to(torch.float32)
    if s.dim() == 2 and s.shape[1] == n_blocks:
        s = s.unsqueeze(2)
    xf = xf * s.to(torch.bfloat16)
    out = xf.reshape(m, n_blocks * block_k)
    if pad:
        out = out[:, :k]
    return out.reshape(m, k).to(torch.bfloat16)


def e8m0_to_float(scale: torch.Tensor) -> torch.Tensor:
    """UE8M0 byte -> 2**(e-127) in FP32; float scales pass through (gemm.py:55-59)."""
    if scale.dtype == torch.uint8:
        return torch.pow(2.0, scale.to(torch.float32) - 127.0)
    return scale.to(torch.float32)


def float_scale_to_e8m0(scale: torch.Tensor) -> torch.Tensor:
    """``clamp(round(log2(s)) + 127, 0, 255)`` as uint8 (gemm.py:62-73)."""
    if scale.dtype == torch.uint8:
        return scale.contiguous()
    s = scale.to(torch.float32)
    tiny = torch.finfo(torch.float32).tiny
    e = torch.round(torch.log2(torch.clamp(s, min=tiny))) + 127.0
    return torch.clamp(e, 0, 255).to(torch.uint8).contiguous()


def dequant_fp4_block(x: torch.Tensor, scale, block_k: int = 32) -> torch.Tensor:
    """Packed E2M1 (+ per-32 scale) -> BF16; follows gemm.py:147-187."""
    if x.dtype in (torch.bfloat16, torch.float16, torch.float32):
        return x.to(torch.bfloat16)
    if x.dtype == torch.int8:
        x = x.view(torch.uint8)
    if x.dtype != torch.uint8:
        return x.to(torch.bfloat16)
    table = torch.from_numpy(E2M1_VALUES).to(x.device)  # the checker also runs on GPU tensors in tests
    low = table[(x & 0x0F).to(torch.long)]
    high = table[((x >> 4) & 0x0F).to(torch.long)]
    out = torch.stack((low, high), dim=-1).flatten(-2)
    if scale is None:
        return out.to(torch.bfloat16)
    k = out.shape[-1]
    n_blocks = (k + block_k - 1) // block_k
    pad = n_blocks * block_k - k
    if pad:
        out = torch.nn.functional.pad(out, (0, pad))
    sf = e8m0_to_float(scale)
    while sf.dim() < out.dim():
        sf = sf.unsqueeze(-2)
    sf = sf.expand(*out.shape[:-1], n_blocks)
    out = out.reshape(*out.shape[:-1], n_blocks, block_k) * sf.unsqueeze(-1)
    out = out.reshape(*out.shape[:-2], n_blocks * block_k)
    if pad:
        out = out[..., :k]
    return out.to(torch.bfloat16)


def reorder_scale_to_sf_atom(scale: np.ndarray) -> np.ndarray:
    """Row-major ``[rows, kb]`` bytes -> 512-byte 128x4 atoms, pad byte 127.

    Byte ``(r, c)`` lands at ``(mt*k_tiles + kt)*512 + m_in_32*16 + m_32*4 + k_in_4``
    with ``mt, m_in_tile = divmod(r, 128)``, ``m_32, m_in_32 = divmod(m_in_tile, 32)``
    and ``kt, k_in_4 = divmod(c, 4)`` (gemm.py:76-116, csrc/cutlass_mxfp8_mxfp4_probe.cu:258-277).
    """
    scale = np.asarray(scale, dtype=np.uint8)
    rows, kb = scale.shape
    m_tiles = (rows + 127) // 128
    k_tiles = (kb + 3) // 4
    padded = np.full((m_tiles * 128, k_tiles * 4), 127, dtype=np.uint8)
    padded[:rows, :kb] = scale
    atoms = padded.reshape(m_tiles, 4, 32, k_tiles, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(atoms).reshape(-1)


def grouped_segments_from_indices(m_indices, m: int, num_groups: int):
    """Per-group row lists for per-row ids or psum ends (gemm.py:303-329)."""
    if m_indices is None:
        if num_groups != 1:
            raise ValueError("m_indices is required when b has multiple groups")
        return [torch.arange(m)]
    if m_indices.numel() == m:
        return [(m_indices == g).nonzero(as_tuple=False).flatten() for g in range(num_groups)]
    if m_indices.numel() == num_groups:
        ends = m_indices.to("cpu").tolist()
        starts = [0] + [int(e) for e in ends[:-1]]
        return [torch.arange(s, int(e)) for s, e in zip(starts, ends)]
    raise ValueError(
        f"m_indices must have length M ({m}) or num_groups ({num_groups}), got {m_indices.numel()}")


def _dequant_fp8_arg(a):
    if isinstance(a, tuple):
        return dequant_fp8_block(a[0], a[1])
    return a.to(torch.bfloat16)


def m_grouped_fp8_fp4_gemm_nt_contiguous(a, b, d: torch.Tensor, m_indices=None) -> None:
    """Oracle for ``m_grouped_fp8_fp4_gemm_nt_contiguous`` (gemm.py:343-367).

    Only the experts that own rows are dequantised (the reference's own
    active-experts variant, gemm.py:411-464, is bit-identical to the fallback
    for per-row ids); the FP32 per-group matmul, the cast to ``d.dtype`` and the
    zero rows are those of gemm.py:357-367.
    """
    a_deq = _dequant_fp8_arg(a)
    b_tensor, b_scale = b if isinstance(b, tuple) else (b, None)
    if b_tensor.dtype == torch.int8:
        b_tensor = b_tensor.view(torch.uint8)
    if b_tensor.dim() == 2:
        w = dequant_fp4_block(b_tensor, b_scale)
        d.copy_(torch.mm(a_deq.to(torch.float32), w.to(torch.float32).t()))
        return
    m, k = a_deq.shape
    num_groups = b_tensor.shape[0]
    d.zero_()
    for g, rows in enumerate(grouped_segments_from_indices(m_indices, m, num_groups)):
        if rows.numel() == 0:
            continue
        sg = None
        if b_scale is not None:
            sg = b_scale[g] if b_scale.dim() == 3 else b_scale
        w = dequant_fp4_block(b_tensor[g], sg)
        if w.shape[-1] != k:
            raise ValueError(f"cannot infer B layout for shape {tuple(w.shape)} and K={k}")
        res = torch.mm(a_deq.index_select(0, rows).to(torch.float32), w.to(torch.float32).t())
        d.index_copy_(0, rows, res.to(d.dtype))


def m_grouped_fp8_fp4_gemm_nt_masked(a, b, d: torch.Tensor, masked_m=None) -> None:
    """Oracle for ``m_grouped_fp8_fp4_gemm_nt_masked`` (gemm.py:529-551).

    ``a`` is ``[G*S, K]`` (G = number of weight groups, S = rows // G); group g
    multiplies rows ``[g*S, g*S + masked_m[g])`` by ``b[g]``, groups in order, so a
    count above S overwrites the next block's rows until that group writes its own;
    every other row of ``d`` is 0.  A 2-D ``b`` (or no ``masked_m``) is one plain
    product over all rows (gemm.py:534-537).
    """
    a_deq = _dequant_fp8_arg(a)
    b_tensor, b_scale = b if isinstance(b, tuple) else (b, None)
    if b_tensor.dtype == torch.int8:
        b_tensor = b_tensor.view(torch.uint8)
    if b_tensor.dim() != 3 or masked_m is None:
        w = dequant_fp4_block(b_tensor, b_scale)
        d.copy_(torch.mm(a_deq.to(torch.float32), w.to(torch.float32).t()))
        return
    num_groups = b_tensor.shape[0]
    block = a_deq.shape[0] // num_groups
    counts = [int(c) for c in masked_m.to("cpu").tolist()]
    d.zero_()
    for g in range(num_groups):
        if counts[g] <= 0:
            continue
        start = g * block
        sg = None
        if b_scale is not None:
            sg = b_scale[g] if b_scale.dim() == 3 else b_scale
        w = dequant_fp4_block(b_tensor[g], sg)
        res = torch.mm(a_deq[start:start + counts[g]].to(torch.float32), w.to(torch.float32).t())
        d[start:start + counts[g]].copy_(res.to(d.dtype))


def transform_weights_for_mega_moe(l1, l2):
    """MegaMoE weight layout (mega.py:14-50) as numpy row permutations.

    L1 rows: the gate half and the up half interleaved in granules of 8 rows
    (mega.py:17-27); scales additionally, per 128-row block, [4 x 32] -> [32 x 4]
    (mega.py:30-39), skipped when the row count is not a multiple of 128.
    """
    def interleave(t):
        g, n = t.shape[:2]
        half = n // 2
        gate = t[:, :half].reshape(g, half // 8, 8, *t.shape[2:])
        up = t[:, half:].reshape(g, half // 8, 8, *t.shape[2:])
        return np.stack([gate, up], axis=2).reshape(t.shape)

    def utccp(t):
        g, n = t.shape[:2]
        if n % 128:
            return t.copy()
        return np.swapaxes(t.reshape(g, n // 128, 4, 32, *t.shape[2:]), 2, 3).reshape(t.shape)

    (w1, s1), (w2, s2) = l1, l2
    return (interleave(w1), utccp(interleave(s1))), (w2.copy(), utccp(s2))


def reference_fp64(a, b, m_indices) -> np.ndarray:
    """Exact product of the quantised operands in FP64 (no BF16 rounding of ``a``).

    Used to show that a kernel is at least as close to the true product as the
    oracle is; this is not a restatement of the reference.
    """
    x, sa = a
    xf = x.to(torch.float32).to(torch.float64)
    m, k = xf.shape
    nb = sa.shape[1]
    bk = k // nb
    xf = (xf.reshape(m, nb, bk) * sa.to(torch.float64).unsqueeze(2)).reshape(m, k)
    bt, bs = b
    bt = bt.view(torch.uint8)
    table = torch.from_numpy(E2M1_VALUES).to(torch.float64)
    out = np.zeros((m, bt.shape[1]), dtype=np.float64)
    ids = m_indices.to(torch.int64)
    for g in torch.unique(ids[(ids >= 0) & (ids < bt.shape[0])]).tolist():
        rows = (ids == g).nonzero().flatten()
        w = torch.stack((table[(bt[g] & 15).long()], table[(bt[g] >> 4).long()]), -1).flatten(-2)
        sf = e8m0_to_float(bs[g]).to(torch.float64)
        w = (w.reshape(w.shape[0], -1, 32) * sf.unsqueeze(-1)).reshape(w.shape[0], -1)
        out[rows.numpy()] = (xf[rows] @ w.t()).numpy()
    return out
