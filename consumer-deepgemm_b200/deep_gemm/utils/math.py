"""Quantisation helpers of the ``deep_gemm.utils.math`` surface.

``ceil_div``, ``align``, ``per_block_cast_to_fp8`` and ``per_token_cast_to_fp8``
keep the reference's semantics (deep_gemm/utils/math.py:7-45 of
lmxxf/Consumer-DeepGEMM): scales are ``amax / 448`` in the dtype of ``x`` and
the payload is ``x / amax * 448`` cast to e4m3.

``per_block_cast_to_fp4`` is new: the reference leaves FP4 quantisation
unimplemented (deep_gemm/utils/math.py:17-18).  It produces OCP MXFP4 weights,
E2M1 elements packed two per byte (low nibble = even k, the order that
consumer_deep_gemm/gemm.py:162-166 decodes) with one UE8M0 scale per 32 values.
All helpers run on any torch device.
"""

from __future__ import annotations

import torch


def ceil_div(a: int, b: int) -> int:
    return (int(a) + int(b) - 1) // int(b)


def align(x: int, alignment: int) -> int:
    return ceil_div(int(x), int(alignment)) * int(alignment)


def per_block_cast_to_fp8(x: torch.Tensor, block_k: int = 128, *args, **kwargs):
    """Per-row, per-``block_k`` FP8 e4m3 quantisation; returns ``(x_fp8, scale)``."""
    fp8_max = torch.finfo(torch.float8_e4m3fn).max
    m, k = x.shape[0], x.shape[1]
    n_blocks = ceil_div(k, block_k)
    pad = n_blocks * block_k - k
    xp = torch.nn.functional.pad(x, (0, pad)) if pad else x
    xb = xp.reshape(m, n_blocks, block_k)
    amax = xb.abs().amax(dim=-1, keepdim=True).clamp(min=1e-12)
    scale = (amax / fp8_max).squeeze(-1)
    xq = (xb / amax * fp8_max).reshape(m, n_blocks * block_k)
    if pad:
        xq = xq[:, :k]
    return xq.to(torch.float8_e4m3fn), scale


def per_token_cast_to_fp8(x: torch.Tensor, *args, **kwargs):
    """Per-row FP8 e4m3 quantisation; returns ``(x_fp8, scale[M, 1])``."""
    fp8_max = torch.finfo(torch.float8_e4m3fn).max
    amax = x.abs().amax(dim=-1, keepdim=True).clamp(min=1e-12)
    return (x / amax * fp8_max).to(torch.float8_e4m3fn), amax / fp8_max


# Round-to-nearest-even decision points between consecutive E2M1 magnitudes
# {0, .5, 1, 1.5, 2, 3, 4, 6}.  A magnitude exactly on a midpoint goes to the
# even code (0, 2, 4 or 6), i.e. the upper neighbour only for 0.75, 1.75 and 3.5.
_E2M1_MID = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
_E2M1_TIE_UP = (False, True, False, True, False, True, False)


def _e2m1_encode(v: torch.Tensor) -> torch.Tensor:
    """FP32 values already divided by their block scale -> 4-bit E2M1 codes."""
    mag = v.abs()
    code = torch.zeros_like(mag, dtype=torch.uint8)
    for mid, up in zip(_E2M1_MID, _E2M1_TIE_UP):
        code += (mag >= mid if up else mag > mid).to(torch.uint8)
    sign = ((v < 0) & (code > 0)).to(torch.uint8) << 3
    return code | sign


def per_block_cast_to_fp4(w: torch.Tensor, block_k: int = 32):
    """OCP MXFP4 quantisation along the last dim.

    Returns ``(packed uint8 [..., K/2], ue8m0 uint8 [..., K/32])``.  The shared
    exponent of a block is ``floor(log2(amax)) - 2`` (E2M1's largest exponent),
    elements are rounded to nearest even and saturate at 6; an all-zero block
    gets scale byte 127.
    """
    if w.shape[-1] % (2 * block_k) and w.shape[-1] % block_k:
        raise ValueError("last dim must be a multiple of the block size")
    shape = w.shape
    k = shape[-1]
    wb = w.to(torch.float32).reshape(*shape[:-1], k // block_k, block_k)
    amax = wb.abs().amax(dim=-1, keepdim=True)
    exp = torch.floor(torch.log2(amax.clamp(min=torch.finfo(torch.float32).tiny))) - 2
    exp = torch.where(amax > 0, exp, torch.zeros_like(exp)).clamp(-127, 127)
    codes = _e2m1_encode(wb / torch.pow(2.0, exp)).reshape(*shape[:-1], k)
    packed = codes[..., 0::2] | (codes[..., 1::2] << 4)
    scale = (exp.squeeze(-1) + 127).to(torch.uint8)
    return packed.contiguous(), scale.contiguous()
