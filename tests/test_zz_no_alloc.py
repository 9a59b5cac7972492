"""The no-allocation entry point (collected last on purpose).

Some callers cannot give the library a workspace: their device memory is already
owned by another allocator, or their host language has no way to reach it.  For
them `cdg_grouped_fp8_fp4_gemm_nt_contiguous_noalloc` uses a 64 MiB scratch
array that lives inside the library.  These tests drive it through the C ABI and
check that two calls in a row give what the regular entry point (caller-owned
workspace) gives -- bit for bit, since both run the same kernels on the same
plan -- and that a problem too large for the scratch is refused before any launch.
"""

import ctypes

import pytest
import torch

import cabi
from conftest import load_gemm_case
from metrics import TOL_NORMWISE, TOL_ROW_L2, errors

pytestmark = pytest.mark.gpu

DEV = "cuda"
CDG_ERR_SCRATCH_TOO_SMALL = 8


def _noalloc():
    fn = cabi.lib().cdg_grouped_fp8_fp4_gemm_nt_contiguous_noalloc
    fn.argtypes = [ctypes.POINTER(cabi.GemmArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _operands(name):
    c = load_gemm_case(name)
    return (c["a"].to(DEV), c["sa"].to(DEV), c["b"].to(DEV), c["sb"].to(DEV), c["m_indices"].to(DEV)), c


def _check_against_regular(name):
    (a, sa, b, sb, ids), c = _operands(name)
    d_ref = torch.empty(c["d"].shape, dtype=torch.bfloat16, device=DEV)
    cabi.gemm(a, sa, b, sb, d_ref, ids)
    d = torch.full(c["d"].shape, float("nan"), dtype=torch.bfloat16, device=DEV)
    g = cabi.make_args(a, sa, b, sb, d, ids)
    st = _noalloc()(ctypes.byref(g), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, cabi.lib().cdg_status_string(st)
    torch.cuda.synchronize()
    out, ref = d.cpu(), d_ref.cpu()
    pad = c["m_indices"] < 0
    assert bool((out[pad].float() == 0).all())
    nw, rl2 = errors(out, ref, ~pad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (name, nw, rl2)
    # the same kernels on the same plan: identical bits, padding rows included
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), name
    # no device wait gave up (the scratch's own status word is private; the library's
    # per-device record covers it)
    assert cabi.device_status() == (0, 0)


def test_noalloc_matches_regular_entry_two_calls_in_a_row():
    _check_against_regular("c0")                    # first call: also resolves the scratch address
    _check_against_regular("edge_aligned_3groups")  # second call reuses the scratch left by the first


def test_noalloc_refuses_problems_larger_than_the_scratch():
    m, k, n, e = 16384, 4096, 128, 1               # activation planes alone need 2*m*k = 128 MiB
    a = torch.empty(m, k, dtype=torch.float8_e4m3fn, device=DEV)
    sa = torch.empty(m, k // 128, dtype=torch.float32, device=DEV)
    b = torch.empty(e, n, k // 2, dtype=torch.uint8, device=DEV)
    sb = torch.empty(e, n, k // 32, dtype=torch.uint8, device=DEV)
    d = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ids = torch.zeros(m, dtype=torch.int32, device=DEV)
    g = cabi.make_args(a, sa, b, sb, d, ids)
    st = _noalloc()(ctypes.byref(g), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == CDG_ERR_SCRATCH_TOO_SMALL
