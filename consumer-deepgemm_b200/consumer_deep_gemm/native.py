"""Loader of the native extension ``consumer_deep_gemm._C`` (binding of libcdg_b200.so).

Mirrors consumer_deep_gemm/native.py of the reference (native.py:13-68): lazy
import, ``is_available``, ``build_info`` and a forwarding
``m_grouped_fp8_fp4_gemm_nt_contiguous`` that returns ``None`` for tensors that
are not on a CUDA device.  Unlike the reference, the GEMM itself never falls back
to Python: ``require()`` raises when the extension is missing.
"""

from __future__ import annotations

from functools import lru_cache


@lru_cache(maxsize=1)
def _load_native():
    try:
        from . import _C  # type: ignore
    except ImportError:
        return None
    return _C


def require():
    """The extension module, or ``RuntimeError`` if it was not built."""
    ext = _load_native()
    if ext is None:
        raise RuntimeError(
            "consumer_deep_gemm._C is not built; run `python consumer-deepgemm_b200/build.py` "
            "(this package has no CPU or Python fallback for the grouped GEMM)")
    return ext


def is_available() -> bool:
    return _load_native() is not None


def build_info() -> dict:
    ext = _load_native()
    if ext is None:
        return {"available": False, "arch": None, "info": None}
    return {
        "available": bool(ext.is_available()),
        "arch": "sm_100a",
        "info": ext.build_info(),
        # names kept from the reference's dict (native.py:34-39); there is no SM120 code here
        "cutlass_sm120_probe": False,
        "cutlass_mxfp8_mxfp4_probe": False,
    }


def _first_tensor(value):
    return value[0] if isinstance(value, tuple) else value


def cutlass_mxfp8_mxfp4_can_implement_probe(a, b, d) -> bool | None:
    """Whether the tensor-core kernel takes these operands (name kept from native.py:42-48)."""
    if not (getattr(a, "is_cuda", False) and getattr(b, "is_cuda", False) and getattr(d, "is_cuda", False)):
        return None
    import torch

    from .gemm import _normalize

    bt = _first_tensor(b)
    ids = torch.zeros(_first_tensor(a).shape[0], dtype=torch.int32, device=d.device) if bt.dim() == 3 else None
    return bool(require().can_implement(*_normalize(a, b, d, ids)) == 1)


def m_grouped_fp8_fp4_gemm_nt_contiguous(*args, **kwargs):
    """Forwarder with the reference's contract: ``None`` unless every operand is on CUDA, else ``True``."""
    if len(args) < 3:
        return None
    a, b, d = _first_tensor(args[0]), _first_tensor(args[1]), args[2]
    if not (getattr(a, "is_cuda", False) and getattr(b, "is_cuda", False) and getattr(d, "is_cuda", False)):
        return None
    from .gemm import m_grouped_fp8_fp4_gemm_nt_contiguous as run

    run(*args, **kwargs)
    return True


def read_device_status(clear: bool = True) -> tuple[int, int]:
    """Device-side errors of the library's kernels on the current device since the last clear.

    Synchronises the device, then returns ``(status, where)``: status 0; 6
    (``CDG_ERR_DEVICE_TIMEOUT``) when a bounded wait gave up -- a GEMM pipeline wait, or a
    wait on another rank's flag in the peer-memory exchange; or 9 (``CDG_ERR_DEVICE_INDEX``)
    when no wait gave up but a kernel skipped an access it could not make (rows that do not
    match their exchange header, a block the planes form cannot run, a misaligned D row
    address) -- and ``where``, the first recorded code (0 when none; layout in
    ``cdg_device_status``).  The GEMM calls themselves
    never synchronise, so a caller that wants to know checks here (after a batch of calls,
    or every call with ``CDG_CHECK_STATUS=1``).
    """
    st, where = require().device_status(bool(clear))
    return int(st), int(where) & 0xFFFFFFFF  # the code's bit pattern (roles >= 8 set the top bit)


def check_device_status() -> None:
    """``read_device_status()``, raising ``RuntimeError`` when a device wait gave up."""
    st, where = read_device_status(True)
    if st:
        what = "a device wait of consumer_deep_gemm gave up" if st == 6 else \
            "a consumer_deep_gemm kernel skipped an access it could not make"
        raise RuntimeError(f"{what} (status {st}, code {where:#010x}); "
                           "the outputs of the calls since the last check are not valid")
