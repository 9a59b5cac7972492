"""Consumer-DeepGEMM for B200: the grouped FP8 x MXFP4 MoE GEMM on sm_100a.

Drop-in for the reference's hot path (``import consumer_deep_gemm as deep_gemm``):
``m_grouped_fp8_fp4_gemm_nt_contiguous`` (and its masked-layout sibling
``m_grouped_fp8_fp4_gemm_nt_masked``) with the same arguments and tensor
layouts, plus the layout and runtime hooks vLLM calls around it
(consumer_deep_gemm/__init__.py:11-48 of the reference, restricted to that path).
"""

from .gemm import m_grouped_fp8_fp4_gemm_nt_contiguous, m_grouped_fp8_fp4_gemm_nt_masked
from .layout import (
    get_mk_alignment_for_contiguous_layout,
    get_mn_major_tma_aligned_tensor,
    get_theoretical_mk_alignment_for_contiguous_layout,
    set_mk_alignment_for_contiguous_layout,
    transform_sf_into_required_layout,
)
from .mega import fp8_fp4_mega_moe, get_symm_buffer_for_mega_moe, transform_weights_for_mega_moe
from .native import build_info as native_build_info
from .native import check_device_status, read_device_status
from .native import is_available as native_is_available
from .utils import get_num_sms, get_pdl, get_tc_util, set_num_sms, set_pdl, set_tc_util

__version__ = "0.2.0"

__all__ = [
    "m_grouped_fp8_fp4_gemm_nt_contiguous",
    "m_grouped_fp8_fp4_gemm_nt_masked",
    "transform_sf_into_required_layout",
    "transform_weights_for_mega_moe",
    "get_symm_buffer_for_mega_moe",
    "fp8_fp4_mega_moe",
    "get_mn_major_tma_aligned_tensor",
    "get_mk_alignment_for_contiguous_layout",
    "set_mk_alignment_for_contiguous_layout",
    "get_theoretical_mk_alignment_for_contiguous_layout",
    "native_build_info",
    "native_is_available",
    "read_device_status",
    "check_device_status",
    "set_num_sms",
    "get_num_sms",
    "set_tc_util",
    "get_tc_util",
    "set_pdl",
    "get_pdl",
]

# Per-call timing of the public functions (CDG_PROFILE=1, reference __init__.py:58-114).
import os as _os

if _os.environ.get("CDG_PROFILE", "0") == "1":
    import sys as _sys

    from . import profile as _profile

    profiler = _profile.install(_sys.modules[__name__])
