"""Grouped FP8 x MXFP4 GEMM with the reference's Python signature.

``m_grouped_fp8_fp4_gemm_nt_contiguous(a, b, d, m_indices=None, **kwargs)``
(reference: consumer_deep_gemm/gemm.py:467-470) computes, for every row ``r``
of ``a`` whose group id ``g = m_indices[r]`` lies in ``[0, G)``::

    d[r, :] = deq(a)[r, :] @ deq(b[g]).T        (FP32 accumulation, cast to d.dtype)

and writes 0 to every other row.  ``deq`` follows the reference's dequant
(gemm.py:31-52, 147-187).  The work runs in libcdg_b200.so on the current CUDA
stream without host synchronisation; this module only normalises the argument
forms the reference accepts and never computes on the host.

Accepted forms (as in the reference):
  a          ``(fp8 [M,K], fp32 [M,K/128])``; ``(fp8 [M,K], int32 [M,ceil(K/512)])`` with UE8M0 scales
             packed four to a word (DeepGEMM's UE8M0 recipe; any strides, e.g. MN-major);
             ``(bf16|fp32 [M,K], any)`` (scale ignored);
             a bare tensor (cast to BF16 like ``a.to(torch.bfloat16)``)
  b          ``(int8|uint8 [G,N,K/2], scale)`` or ``[N,K/2]`` for one group; scale is
             uint8/float8_e8m0fnu UE8M0 ``[G,N,K/32]``, a float ``[G,N,K/32]``, the
             int32 output of ``transform_sf_into_required_layout``, or absent (1.0)
  m_indices  int32/int64 per-row ids (-1 = padding), psum ends (length G), or None (G == 1)
  kwargs     ``recipe_a=(1,128)``, ``recipe_b=(1,32)``, ``disable_ue8m0_cast`` (accepted;
             the FP32 activation scales are always used exactly).  Library-internal ones:
             ``_skip_ungrouped_rows`` (leave rows outside every group unwritten),
             ``_round_weight_scales`` (float weight scales rounded to powers of two),
             ``_force_exact_path`` (the SIMT kernel), ``_d_rows`` (int64 [M] device
             addresses: row r of D is stored at ``_d_rows[r]``, 0 = not stored; ``d`` then
             only gives the shape, e.g. an expanded [1, N] BF16 view)
"""

from __future__ import annotations

import torch

import os

from . import native

# CDG_CHECK_STATUS=1: synchronise after every call and raise if a device wait gave up (a
# debugging aid; the calls otherwise never wait for the device).
_CHECK_STATUS = os.environ.get("CDG_CHECK_STATUS", "0") == "1"

__all__ = ["m_grouped_fp8_fp4_gemm_nt_contiguous", "m_grouped_fp8_fp4_gemm_nt_masked"]

_FLOAT_SCALES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)


def _normalize(a, b, d, m_indices):
    """Map the reference's argument forms onto ``_C.grouped_gemm``'s tensors."""
    if isinstance(a, tuple):
        if len(a) != 2:
            raise ValueError("a must be a (tensor, scale) tuple")
        x, sa = a
        if x.dtype == torch.float8_e4m3fn:
            if sa is None:
                raise ValueError("FP8 a needs its scale")
            if sa.dim() != 2 or sa.shape[0] != x.shape[0]:
                raise ValueError(f"a scale must be [M, K/128], got {tuple(sa.shape)}")
            if sa.dtype != torch.int32:  # int32: UE8M0 scales packed four to a word
                sa = sa.float() if sa.dtype != torch.float32 else sa
        elif x.dtype in (torch.bfloat16, torch.float32):
            sa = None  # the reference passes BF16/FP32 activations through unscaled (gemm.py:33-34)
        else:
            raise ValueError(f"a must be FP8/BF16/FP32, got {x.dtype}")
    else:
        x, sa = a, None
        if x.dtype == torch.float8_e4m3fn:
            # bare FP8 is cast to BF16 without a scale (gemm.py:289-293): scale 1 is exact
            sa = torch.ones(x.shape[0], (x.shape[1] + 127) // 128, dtype=torch.float32, device=x.device)
        elif x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
    if isinstance(b, tuple):
        if len(b) != 2:
            raise ValueError("b must be a (tensor, scale) tuple")
        bt, bs = b
    else:
        bt, bs = b, None
    if bt.dtype not in (torch.int8, torch.uint8):
        raise NotImplementedError(f"b must be packed FP4 (int8/uint8), got {bt.dtype}")
    single = bt.dim() == 2
    if single:
        bt = bt.unsqueeze(0)
        if bs is not None and bs.dim() == 2:
            bs = bs.unsqueeze(0)
        m_indices = None  # one group: every row uses it (gemm.py:347-350)
    if bt.dim() != 3:
        raise ValueError(f"grouped B must be 2D or 3D, got shape {tuple(bt.shape)}")
    bt = bt.view(torch.uint8)
    k = x.shape[1]
    if bs is None:
        bs = torch.full((bt.shape[0], bt.shape[1], (k + 31) // 32), 127, dtype=torch.uint8, device=bt.device)
    elif bs.dtype == torch.float8_e8m0fnu:
        bs = bs.view(torch.uint8)
    elif bs.dtype in _FLOAT_SCALES:
        bs = bs.float() if bs.dtype != torch.float32 else bs
    elif bs.dtype not in (torch.uint8, torch.int32):
        raise ValueError(f"b scale must be UE8M0 bytes, float or transformed int32, got {bs.dtype}")
    if bs.dtype != torch.int32 and bs.dim() != 3:
        raise ValueError(f"b scale must be [G, N, K/32], got {tuple(bs.shape)}")
    if m_indices is None and bt.shape[0] != 1:
        raise ValueError("m_indices is required when b has multiple groups")
    if bs.dtype != torch.int32 and bt.shape[1] % 128 == 0 and k % 128 == 0 and bt.shape[0] * bt.shape[1] >= 65536:
        _warn_row_major_scales(bs)
    return x, sa, bt, bs, d, m_indices


_warned_row_major = False


def _warn_row_major_scales(bs):
    """Once per process: weight scales that arrive row-major are reordered into tensor-core atoms
    inside every call (a read of all experts' scales, ~0.5 ms at E=256, N=K=4096), where
    ``transform_sf_into_required_layout`` does it once at weight load."""
    global _warned_row_major
    if _warned_row_major:
        return
    _warned_row_major = True
    import warnings

    warnings.warn("consumer_deep_gemm: weight scales passed row-major (%s); every call reorders them for the "
                  "tensor cores. Pass transform_sf_into_required_layout(scale) (done once at weight load) "
                  "instead." % str(bs.dtype).replace("torch.", ""), RuntimeWarning, stacklevel=4)


def _check_recipes(kwargs):
    ra = kwargs.get("recipe_a")
    rb = kwargs.get("recipe_b")
    if ra is not None and tuple(ra) != (1, 128):
        raise NotImplementedError(f"recipe_a {tuple(ra)} is not supported; this kernel takes (1, 128)")
    if rb is not None and tuple(rb) != (1, 32):
        raise NotImplementedError(f"recipe_b {tuple(rb)} is not supported; this kernel takes (1, 32)")


def m_grouped_fp8_fp4_gemm_nt_contiguous(a, b, d, m_indices=None, **kwargs) -> None:
    """M-grouped FP8 x FP4 GEMM for the MoE contiguous layout (see module docstring)."""
    _check_recipes(kwargs)
    x, sa, bt, bs, d, ids = _normalize(a, b, d, m_indices)
    flags = ((1 if kwargs.get("_force_exact_path") else 0) | (4 if kwargs.get("_skip_ungrouped_rows") else 0) |
             (8 if kwargs.get("_round_weight_scales") else 0))
    native.require().grouped_gemm(x, sa, bt, bs, d, ids, flags, False, kwargs.get("_d_rows"))
    if _CHECK_STATUS:
        native.check_device_status()


def _flatten_groups(t):
    """[G, S, ...] -> [G*S, ...] (a view when the tensor allows one)."""
    if t is None or t.dim() != 3:
        return t
    return t.reshape(t.shape[0] * t.shape[1], t.shape[2])


def m_grouped_fp8_fp4_gemm_nt_masked(a, b, d, masked_m=None, **kwargs) -> None:
    """M-grouped FP8 x FP4 GEMM, masked layout (reference: consumer_deep_gemm/gemm.py:529-551).

    ``a`` holds G blocks of S rows, as ``[G*S, K]`` (the reference's form) or
    ``[G, S, K]``; ``d`` is ``[G*S, N]`` or ``[G, S, N]`` alike.  Group g multiplies
    rows ``[g*S, g*S + masked_m[g])`` by ``b[g]``; every other row of ``d`` is 0.
    With a 2-D ``b`` every row is multiplied by it and ``masked_m`` is not used.
    ``masked_m`` (int32/int64 ``[G]``) is read on the device, so the call does not
    synchronise with the host.  ``expected_m`` (a scheduling hint in DeepGEMM's
    signature) is accepted and not needed.
    """
    _check_recipes(kwargs)
    if isinstance(a, tuple):
        if len(a) != 2:
            raise ValueError("a must be a (tensor, scale) tuple")
        a = (_flatten_groups(a[0]), _flatten_groups(a[1]))
    else:
        a = _flatten_groups(a)
    d2 = d
    if d.dim() == 3:
        try:
            d2 = d.view(d.shape[0] * d.shape[1], d.shape[2])
        except RuntimeError as exc:
            raise ValueError("a 3-D d must be viewable as [G*S, N]") from exc
    single = (b[0] if isinstance(b, tuple) else b).dim() == 2
    if masked_m is None and not single:
        raise ValueError("masked_m is required when b has multiple groups")
    x, sa, bt, bs, d2, _ = _normalize(a, b, d2, masked_m)
    if single:
        ids, masked = None, False
    else:
        if masked_m.dim() != 1 or masked_m.numel() != bt.shape[0]:
            raise ValueError(f"masked_m must be [G] with G = {bt.shape[0]}, got {tuple(masked_m.shape)}")
        if masked_m.dtype not in (torch.int32, torch.int64):
            masked_m = masked_m.to(torch.int32)
        ids = masked_m.to(x.device).contiguous()
        masked = True
    flags = 1 if kwargs.get("_force_exact_path") else 0
    native.require().grouped_gemm(x, sa, bt, bs, d2, ids, flags, masked)
    if _CHECK_STATUS:
        native.check_device_status()
