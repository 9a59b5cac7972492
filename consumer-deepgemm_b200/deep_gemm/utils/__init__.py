"""``deep_gemm.utils`` compatibility surface."""

from . import math  # noqa: F401
from .math import align, ceil_div, per_block_cast_to_fp4, per_block_cast_to_fp8, per_token_cast_to_fp8  # noqa: F401
