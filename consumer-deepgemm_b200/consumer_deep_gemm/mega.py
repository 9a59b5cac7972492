"""MegaMoE entry points of the reference (consumer_deep_gemm/mega.py:1-81).

``transform_weights_for_mega_moe`` is pure weight-layout work and runs here as a
device row gather (libcdg_b200.so ``cdg_mega_moe_transform_rows``):

* L1 (gate/up) weights and scales: the gate half and the up half of the N rows are
  interleaved in granules of 8 rows (mega.py:14-27);
* scales of both layers: each 128-row block is transposed as [4 x 32] -> [32 x 4], the
  row order tcgen05.cp's 32x128b.warpx4 pattern loads (mega.py:30-39); tensors whose row
  count is not a multiple of 128 are returned unchanged, as in the reference.

The fused distributed MegaMoE kernel is not part of the reference either: the two
entry points below raise NotImplementedError exactly as the reference's do.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import native

_INTERLEAVE, _UTCCP = 1, 2


def _rows(t: torch.Tensor, kind: int) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError("transform_weights_for_mega_moe runs on the GPU (libcdg_b200.so)")
    if kind & _UTCCP and t.shape[1] % 128 != 0:
        kind &= ~_UTCCP
        if kind == 0:
            return t.contiguous()
    return native.require().mega_moe_transform_rows(t, kind)


def transform_weights_for_mega_moe(
    l1_weights: Tuple[torch.Tensor, torch.Tensor],
    l2_weights: Tuple[torch.Tensor, torch.Tensor],
) -> Tuple[Tuple[torch.Tensor, torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]:
    """((L1 weights, L1 scales), (L2 weights, L2 scales)) in the MegaMoE layout (mega.py:42-50)."""
    w1, s1 = l1_weights
    w2, s2 = l2_weights
    return (
        (_rows(w1, _INTERLEAVE), _rows(s1, _INTERLEAVE | _UTCCP)),
        (w2.contiguous(), _rows(s2, _UTCCP)),
    )


def get_symm_buffer_for_mega_moe(*args, **kwargs):
    raise NotImplementedError(
        "The distributed MegaMoE symmetric buffer is not implemented (neither is it in the reference); "
        "use the grouped GEMM path (consumer_deep_gemm.moe.MoELayer) instead.")


def fp8_fp4_mega_moe(y: torch.Tensor, l1_weights, l2_weights, sym_buffer,
                     cumulative_local_expert_recv_stats: Optional[torch.Tensor] = None,
                     recipe: Tuple[int, int, int] = (1, 1, 32), activation: str = "swiglu",
                     activation_clamp: Optional[float] = None, fast_math: bool = True):
    raise NotImplementedError(
        "fp8_fp4_mega_moe is not implemented (neither is it in the reference); "
        "use consumer_deep_gemm.moe.MoELayer instead.")
