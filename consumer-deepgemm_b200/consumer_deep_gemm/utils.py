"""Runtime knobs of the DeepGEMM API (reference: consumer_deep_gemm/utils.py:1-50).

Two of them reach the kernels of libcdg_b200.so:

* ``set_num_sms(n)`` limits the persistent GEMM kernels to ``n`` SMs (0 = all), e.g. to
  leave SMs free for kernels that overlap the GEMM on another stream
  (``cdg_set_num_sms``); ``get_num_sms()`` reports the limit, or the device's SM count.
* ``set_pdl(v)`` chooses whether the GEMM's kernels after the first are launched with
  programmatic stream serialization (``cdg_set_pdl``; on by default in this build, where
  every kernel waits for its predecessor on the device).

The reference stores all of these without reading them.  ``set_tc_util``,
``set_ignore_compile_dims`` and ``set_block_size_multiple_of`` tune DeepGEMM's JIT
kernel selection, which has no counterpart here; they are kept so that callers of the
DeepGEMM API run unchanged, and their values are only stored.
"""

from __future__ import annotations

import torch

from . import native

_stored = {"tc_util": 1.0, "ignore_compile_dims": False, "block_size_multiple_of": 1}


def set_num_sms(num_sms: int) -> None:
    n = int(num_sms)
    if n < 0:
        raise ValueError("num_sms must be >= 0 (0 = all SMs)")
    native.require().set_num_sms(n)


def get_num_sms() -> int:
    if native.is_available():
        n = int(native.require().get_num_sms())
        if n > 0:
            return n
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def set_pdl(v: bool) -> None:
    native.require().set_pdl(bool(v))


def get_pdl() -> bool:
    return bool(native.require().get_pdl()) if native.is_available() else True


def set_tc_util(tc_util: float) -> None:
    _stored["tc_util"] = float(tc_util)


def get_tc_util() -> float:
    return _stored["tc_util"]


def set_ignore_compile_dims(v: bool) -> None:
    _stored["ignore_compile_dims"] = bool(v)


def set_block_size_multiple_of(v: int) -> None:
    _stored["block_size_multiple_of"] = int(v)
