"""Shared pytest set-up: import paths, the ``gpu`` marker and golden-fixture loading."""

import glob
import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "consumer-deepgemm_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


_DTYPES = {
    "torch.float8_e4m3fn": (np.uint8, torch.float8_e4m3fn),
    "torch.bfloat16": (np.int16, torch.bfloat16),
    "torch.float32": (np.float32, torch.float32),
    "torch.uint8": (np.uint8, torch.uint8),
    "torch.int8": (np.int8, torch.int8),
}


def to_torch(arr: np.ndarray, dtype_name: str) -> torch.Tensor:
    """Rebuild a tensor stored as a raw integer view by ``make_golden.py``."""
    _, tdtype = _DTYPES[dtype_name]
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if tdtype in (torch.float8_e4m3fn, torch.bfloat16):
        return t.view(tdtype)
    return t.to(tdtype)


def load_gemm_case(name: str) -> dict:
    """Inputs and reference output of one golden GEMM case, as CPU tensors."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    case = {
        "a": to_torch(z["a"], str(z["a_dtype"])),
        "b": torch.from_numpy(z["b"].astype(np.uint8)),
        "sb": to_torch(z["sb"], str(z["sb_dtype"])),
        "d": to_torch(z["d"], str(z["d_dtype"])),
        "d_dtype": _DTYPES[str(z["d_dtype"])][1],
        "m_indices": torch.from_numpy(z["m_indices"]) if bool(z["has_m_indices"]) else None,
        "masked": bool(z["masked"]) if "masked" in z.files else False,
    }
    case["sa"] = torch.from_numpy(z["sa"]) if "sa" in z.files else None
    case["sa_packed"] = torch.from_numpy(z["sa_packed"]) if "sa_packed" in z.files else None
    return case


GEMM_CASES = sorted(
    os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
    if os.path.basename(p).startswith(("kat_", "edge_", "c0")))

PACKED_SCALE_CASES = sorted(
    os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "ue8m0x4_*.npz")))

MASKED_CASES = sorted(
    os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "masked_*.npz")))


@pytest.fixture(params=GEMM_CASES)
def gemm_case(request):
    c = load_gemm_case(request.param)
    c["name"] = request.param
    return c
