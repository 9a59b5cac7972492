"""``import deep_gemm`` alias for the B200 build of Consumer-DeepGEMM (deep_gemm/__init__.py:1-3)."""

from consumer_deep_gemm import *  # noqa: F401,F403
from consumer_deep_gemm import __all__  # noqa: F401
from . import utils  # noqa: F401
