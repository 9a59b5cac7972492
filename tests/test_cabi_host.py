"""CPU-side checks of the C ABI: the library loads, exports what the header declares,
and its host-only entry points validate arguments (nothing here touches a GPU)."""

import ctypes

import pytest
import torch

import cabi


def test_library_exports_every_declared_symbol():
    names = cabi.declared_functions()
    assert "cdg_grouped_fp8_fp4_gemm_nt_contiguous" in names and len(names) >= 9
    lib = cabi.lib()
    for n in names:
        assert hasattr(lib, n), n


def test_build_info_and_alignment():
    lib = cabi.lib()
    assert b"sm_100a" in lib.cdg_build_info()
    assert lib.cdg_mk_alignment_for_contiguous_layout() == 128
    assert lib.cdg_status_string(0) == b"ok"


class _Fake:
    """Tensor stand-in with a fake device address, for host-only argument checks."""

    def __init__(self, shape, dtype, addr=1 << 20):
        self.shape = shape
        self.dtype = dtype
        self._addr = addr
        st, acc = [], 1
        for s in reversed(shape):
            st.append(acc)
            acc *= s
        self._strides = tuple(reversed(st))

    def data_ptr(self):
        return self._addr

    def stride(self, i):
        return self._strides[i]

    def numel(self):
        n = 1
        for s in self.shape:
            n *= s
        return n


def _args(M=256, N=256, K=512, E=4, a_dtype=torch.float8_e4m3fn, d_dtype=torch.bfloat16, sb_dtype=torch.uint8,
          ids_len=None, addr=1 << 20):
    a = _Fake((M, K), a_dtype, addr)
    sa = _Fake((M, (K + 127) // 128), torch.float32, addr)
    b = _Fake((E, N, K // 2), torch.uint8, addr)
    sb = _Fake((E, N, K // 32), sb_dtype, addr)
    d = _Fake((M, N), d_dtype, addr)
    ids = _Fake((ids_len if ids_len is not None else M,), torch.int32, addr)
    return cabi.make_args(a, sa, b, sb, d, ids)


def test_can_implement_envelope():
    lib = cabi.lib()
    ok = _args()
    assert lib.cdg_can_implement(ctypes.byref(ok)) == 1
    assert lib.cdg_can_implement(ctypes.byref(_args(N=200))) == 0          # N not a multiple of 128
    assert lib.cdg_can_implement(ctypes.byref(_args(K=192))) == 0          # K not a multiple of 128 (sa cols 1)
    assert lib.cdg_can_implement(ctypes.byref(_args(a_dtype=torch.bfloat16))) == 0
    assert lib.cdg_can_implement(ctypes.byref(_args(d_dtype=torch.float32))) == 0
    # float32 weight scales: the tensor-core kernels take them (as UE8M0 codes when all are powers
    # of two, which the device decides per call; the exact SIMT kernel otherwise)
    assert lib.cdg_can_implement(ctypes.byref(_args(sb_dtype=torch.float32))) == 1
    assert lib.cdg_can_implement(ctypes.byref(_args(addr=(1 << 20) + 8))) == 0   # misaligned operands
    bad = _args(ids_len=7)                                                  # neither M nor E long
    assert lib.cdg_can_implement(ctypes.byref(bad)) == -1
    assert lib.cdg_grouped_fp8_fp4_workspace_bytes(ctypes.byref(bad)) == 0


def test_row_table_output_arguments():
    """cdg_gemm_args.d_rows (ABI 2): a row table replaces `d` (which may then be NULL) for a BF16
    output only; without either there is no output."""
    lib = cabi.lib()
    assert ctypes.sizeof(cabi.GemmArgs) == cabi.GemmArgs.d_rows.offset + 8  # the last field, as in the header
    g = _args()
    g.d_rows, g.d = 1 << 21, None
    assert lib.cdg_can_implement(ctypes.byref(g)) == 1
    g = _args(d_dtype=torch.float32)
    g.d_rows = 1 << 21
    assert lib.cdg_can_implement(ctypes.byref(g)) == -1
    g = _args()
    g.d = None
    assert lib.cdg_can_implement(ctypes.byref(g)) == -1
    assert lib.cdg_status_string(9) != lib.cdg_status_string(6)  # skipped access vs wait timeout


def test_workspace_size_covers_activation_planes():
    lib = cabi.lib()
    g = _args(M=1000, N=256, K=512, E=4)
    nbytes = lib.cdg_grouped_fp8_fp4_workspace_bytes(ctypes.byref(g))
    nblk = (1000 + 127) // 128
    # activation planes (hi, lo), per-row exponents, weight scale atoms transformed per call
    assert nbytes >= 2 * nblk * 128 * 512 + nblk * 128 * 4 + 4 * 2 * 4 * 512


def test_invalid_arguments_rejected_before_launch():
    lib = cabi.lib()
    g = _args()
    st = lib.cdg_grouped_fp8_fp4_gemm_nt_contiguous(ctypes.byref(g), None, 0, None)
    assert st != 0  # no workspace (or no device): refused on the host, nothing launched
    g2 = _args(ids_len=5)
    assert lib.cdg_grouped_fp8_fp4_gemm_nt_contiguous(ctypes.byref(g2), None, 0, None) == 1


def test_sf_atoms_bytes():
    lib = cabi.lib()
    assert lib.cdg_sf_atoms_bytes(256, 4096, 128) == 256 * 32 * 32 * 512
    assert lib.cdg_sf_atoms_bytes(1, 300, 10) == 3 * 3 * 512
    assert lib.cdg_sf_atoms_bytes(0, 1, 1) == 0


def test_quantising_entry_points_validate_scale_format_and_topk():
    """scale_fmt outside {CDG_SCALE_FP32, CDG_SCALE_POW2} and the one-rank dispatch's limits are
    refused on the host, before anything is launched (fake device addresses)."""
    lib = cabi.lib()
    P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    lib.cdg_quant_fp8_rows.argtypes = [P, I32, I64, I64, I64, P, I64, P, I64, I64, I32, P]
    lib.cdg_silu_mul_quant_fp8.argtypes = [P, I64, I64, I64, P, P, I64, P, I64, I64, I32, P]
    lib.cdg_ep_quant_dispatch_local.argtypes = [P, I32, I64, P, I32, I64, I64, I64, I64, P, P, P, P, P, I64, P, P,
                                                I32, P]
    x = P(1 << 20)
    bf16, i32 = cabi.DT["bf16"], cabi.DT["i32"]
    invalid = 1  # CDG_ERR_INVALID_ARGUMENT
    assert lib.cdg_quant_fp8_rows(x, bf16, 512, 4, 512, x, 512, x, 4, 1, 2, None) == invalid
    assert lib.cdg_silu_mul_quant_fp8(x, 1024, 4, 512, None, x, 512, x, 4, 1, -1, None) == invalid
    # topk above 32, then a bad scale format
    assert lib.cdg_ep_quant_dispatch_local(x, bf16, 512, x, i32, 4, 33, 8, 512, x, x, x, x, x, 1024, x, x, 0,
                                           None) == invalid
    assert lib.cdg_ep_quant_dispatch_local(x, bf16, 512, x, i32, 4, 8, 8, 512, x, x, x, x, x, 1024, x, x, 7,
                                           None) == invalid
    # K not a multiple of 128
    assert lib.cdg_quant_fp8_rows(x, bf16, 500, 4, 500, x, 500, x, 4, 1, 0, None) == invalid
