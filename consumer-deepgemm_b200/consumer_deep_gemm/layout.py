"""Scale-factor layout hooks of the DeepGEMM API (reference: consumer_deep_gemm/layout.py).

``transform_sf_into_required_layout`` is where weight scales get the layout the
tensor cores read, once, at weight-load time.  The reference makes it a no-op
(layout.py:6-19) and instead reorders lazily inside every launch, caching by
data pointer (csrc/cutlass_mxfp8_mxfp4_probe.cu:349-385).  Here it runs the
sm_100a kernel ``cdg_sf_atom_kernel`` over all experts in one launch and returns
an int32 tensor ``[G, N/128, K/128, 128]`` of 512-byte 128x4 atoms (the
128x4 reorder of gemm.py:76-116, applied per expert), which the GEMM recognises
by its dtype and shape.  Float weight scales that are all powers of two (an MXFP4
checkpoint's scales stored as float) become the same atoms, exactly; other float
scales are returned unchanged (the GEMM then keeps them exact on its SIMT path).
Activation scales (``is_sfa=True``) stay FP32 and are returned unchanged: the GEMM
applies them exactly.
"""

from __future__ import annotations

import torch

from . import native

_mk_alignment_for_contiguous_layout = 128


def transform_sf_into_required_layout(sf: torch.Tensor, mn=None, k=None, recipe=None, num_groups=None,
                                      is_sfa: bool = False, *args, **kwargs) -> torch.Tensor:
    """Weight scales ``[G, N, K/32]`` (UE8M0 bytes) -> tensor-core atoms; anything else unchanged.

    Accepts both call forms vLLM uses: ``(sf, mn=..., k=..., recipe=..., num_groups=..., is_sfa=...)``
    and ``(sf, m, n, recipe, num_groups)``.
    """
    if is_sfa or not isinstance(sf, torch.Tensor) or not sf.is_cuda:
        return sf
    if sf.dtype == torch.float8_e8m0fnu:
        sf = sf.view(torch.uint8)
    if sf.dtype in (torch.float32, torch.float16, torch.bfloat16):
        codes = _exact_ue8m0(sf)
        if codes is None:
            return sf
        sf = codes
    if sf.dtype != torch.uint8:
        return sf
    if sf.dim() == 2:
        sf = sf.unsqueeze(0)
    if sf.dim() != 3:
        return sf
    n, kb = sf.shape[1], sf.shape[2]
    if n % 128 or kb % 4:
        return sf  # outside the tensor-core envelope: the exact SIMT path reads row-major scales
    return native.require().transform_sf_atoms(sf)


def _exact_ue8m0(sf: torch.Tensor):
    """UE8M0 bytes of float scales that are all powers of two 2^(c-127), c in [0, 254]
    (c = the FP32 exponent field; 2^-127 is code 0), else None.  Reads one bool back to the
    host: a weight-load-time synchronisation."""
    bits = sf.float().contiguous().view(torch.int32)
    ex = (bits >> 23) & 0xFF
    tiny = bits == 0x00400000
    exact = ((bits & 0x807FFFFF) == 0) & (ex >= 1) & (ex <= 254) | tiny
    if not bool(exact.all()):
        return None
    return torch.where(tiny, torch.zeros_like(ex), ex).to(torch.uint8)


def get_mn_major_tma_aligned_tensor(x: torch.Tensor) -> torch.Tensor:
    """Contiguous view (the kernel reads activation scales with arbitrary strides)."""
    return x if x.is_contiguous() else x.contiguous()


def get_mk_alignment_for_contiguous_layout() -> int:
    """Row alignment of each group in the contiguous layout (layout.py:32-34)."""
    return _mk_alignment_for_contiguous_layout


def set_mk_alignment_for_contiguous_layout(alignment: int) -> None:
    global _mk_alignment_for_contiguous_layout
    _mk_alignment_for_contiguous_layout = int(alignment)


def get_theoretical_mk_alignment_for_contiguous_layout(*args, **kwargs) -> int:
    return 1
