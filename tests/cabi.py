"""ctypes binding of include/cdg_b200.h, the way a non-Python host would bind the library.

The GPU parity tests drive the kernels through this C ABI (not through the
torch extension) so that what is checked is the boundary a foreign caller sees.
"""

from __future__ import annotations

import ctypes
import os
import re

import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(REPO, "consumer-deepgemm_b200", "consumer_deep_gemm", "libcdg_b200.so")
HEADER = os.path.join(REPO, "include", "cdg_b200.h")

CDG_OK = 0
DT = {"e4m3": 1, "bf16": 2, "f32": 3, "ue8m0": 4, "i32": 5, "i64": 6, "ue8m0_x4": 7}
SF_ROW_MAJOR, SF_ATOMS = 0, 1
INDEX_PER_ROW, INDEX_PSUM, INDEX_NONE, INDEX_MASKED = 0, 1, 2, 3
FLAG_FORCE_GENERIC = 1
FLAG_SINGLE_CTA = 2
FLAG_ROUND_SFB = 8


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p), ("a_dtype", ctypes.c_int32), ("a_row_stride", ctypes.c_int64),
        ("sa", ctypes.c_void_p), ("sa_stride_m", ctypes.c_int64), ("sa_stride_k", ctypes.c_int64),
        ("sa_cols", ctypes.c_int32),
        ("b", ctypes.c_void_p), ("b_stride_e", ctypes.c_int64), ("b_stride_n", ctypes.c_int64),
        ("sfb", ctypes.c_void_p), ("sfb_dtype", ctypes.c_int32), ("sfb_layout", ctypes.c_int32),
        ("sfb_stride_e", ctypes.c_int64), ("sfb_stride_n", ctypes.c_int64),
        ("m_indices", ctypes.c_void_p), ("m_indices_dtype", ctypes.c_int32), ("index_form", ctypes.c_int32),
        ("m_indices_len", ctypes.c_int64),
        ("d", ctypes.c_void_p), ("d_dtype", ctypes.c_int32), ("d_row_stride", ctypes.c_int64),
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64), ("E", ctypes.c_int64),
        ("flags", ctypes.c_int32), ("sa_dtype", ctypes.c_int32),
        ("d_rows", ctypes.c_void_p),
    ]


def declared_functions() -> list[str]:
    """Names of the functions include/cdg_b200.h declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(cdg_[a-z_0-9]+)\s*\(", text, re.M)))


_lib = None


def lib():
    global _lib
    if _lib is None:
        l = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER(GemmArgs)
        l.cdg_grouped_fp8_fp4_gemm_nt_contiguous.argtypes = [P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        l.cdg_grouped_fp8_fp4_gemm_nt_masked.argtypes = [P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        l.cdg_grouped_fp8_fp4_workspace_bytes.argtypes = [P]
        l.cdg_grouped_fp8_fp4_workspace_bytes.restype = ctypes.c_size_t
        l.cdg_can_implement.argtypes = [P]
        l.cdg_transform_sf.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        l.cdg_sf_atoms_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        l.cdg_sf_atoms_bytes.restype = ctypes.c_size_t
        l.cdg_read_device_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        l.cdg_device_status.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
        l.cdg_ep_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
        l.cdg_set_num_sms.argtypes = [ctypes.c_int32]
        l.cdg_set_pdl.argtypes = [ctypes.c_int32]
        l.cdg_build_info.restype = ctypes.c_char_p
        l.cdg_status_string.restype = ctypes.c_char_p
        _lib = l
    return _lib


def _code(t: torch.Tensor) -> int:
    return {torch.float8_e4m3fn: DT["e4m3"], torch.bfloat16: DT["bf16"], torch.float32: DT["f32"],
            torch.uint8: DT["ue8m0"], torch.int32: DT["i32"], torch.int64: DT["i64"]}[t.dtype]


def make_args(a, sa, b, sb, d, m_indices, flags=0, sb_atoms=False, masked=False, d_rows=None) -> GemmArgs:
    g = GemmArgs()
    M, K = a.shape
    E, N = b.shape[0], b.shape[1]
    g.a, g.a_dtype, g.a_row_stride = a.data_ptr(), _code(a), a.stride(0)
    if sa is not None:
        g.sa, g.sa_stride_m, g.sa_stride_k, g.sa_cols = sa.data_ptr(), sa.stride(0), sa.stride(1), sa.shape[1]
        g.sa_dtype = DT["ue8m0_x4"] if sa.dtype == torch.int32 else DT["f32"]
    g.b, g.b_stride_e, g.b_stride_n = b.data_ptr(), b.stride(0), b.stride(1)
    g.sfb = sb.data_ptr()
    if sb_atoms:
        g.sfb_dtype, g.sfb_layout = DT["ue8m0"], SF_ATOMS
    else:
        g.sfb_dtype, g.sfb_layout = _code(sb), SF_ROW_MAJOR
        g.sfb_stride_e, g.sfb_stride_n = sb.stride(0), sb.stride(1)
    if m_indices is None:
        g.index_form = INDEX_NONE
    else:
        g.m_indices, g.m_indices_dtype, g.m_indices_len = m_indices.data_ptr(), _code(m_indices), m_indices.numel()
        g.index_form = INDEX_MASKED if masked else INDEX_PER_ROW if m_indices.numel() == M else INDEX_PSUM
    g.d, g.d_dtype, g.d_row_stride = d.data_ptr(), _code(d), d.stride(0)
    if d_rows is not None:  # rows stored through the table; `d` only gives dtype and width
        g.d_rows, g.d, g.d_row_stride = d_rows.data_ptr(), None, N
    g.M, g.N, g.K, g.E, g.flags = M, N, K, E, flags
    return g


def gemm(a, sa, b, sb, d, m_indices, flags=0, sb_atoms=False, stream=None, check_status=True, masked=False,
         d_rows=None):
    """Run the GEMM through the C ABI on `stream` (default: torch's current stream).

    masked=True: `m_indices` is masked_m [G] and the masked entry point runs.
    d_rows: int64 [M] device addresses of D's rows (cdg_gemm_args.d_rows)."""
    l = lib()
    g = make_args(a, sa, b, sb, d, m_indices, flags, sb_atoms, masked, d_rows)
    nbytes = l.cdg_grouped_fp8_fp4_workspace_bytes(ctypes.byref(g))
    assert nbytes > 0, "invalid arguments"
    ws = torch.empty(nbytes + 1024, dtype=torch.uint8, device=d.device)
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    s = stream if stream is not None else torch.cuda.current_stream(d.device)
    entry = l.cdg_grouped_fp8_fp4_gemm_nt_masked if masked else l.cdg_grouped_fp8_fp4_gemm_nt_contiguous
    st = entry(ctypes.byref(g), ctypes.c_void_p(base), nbytes, ctypes.c_void_p(s.cuda_stream))
    if st != CDG_OK:
        raise RuntimeError(f"cdg status {st}: {l.cdg_status_string(st).decode()}")
    if check_status:
        st = l.cdg_read_device_status(ctypes.c_void_p(base), ctypes.c_void_p(s.cuda_stream))
        if st != CDG_OK:
            off = base - ws.data_ptr()
            where = int(ws[off + 36:off + 40].cpu().view(torch.int32)[0])  # control word 9
            raise RuntimeError(f"device status {st}: {l.cdg_status_string(st).decode()}; wait code {where:#010x}")
    return ws


# Block classes of the prep kernel, in the order of their control words (1..6).
BLOCK_CLASSES = ("tiny", "narrow", "wide", "zero", "irregular", "wide_direct")


def block_classes(ws: torch.Tensor) -> dict:
    """Blocks per class planned by the call that used workspace `ws` (as returned by gemm)."""
    off = (ws.data_ptr() + 1023) // 1024 * 1024 - ws.data_ptr()
    words = ws[off + 4:off + 4 + 4 * len(BLOCK_CLASSES)].cpu().view(torch.int32).tolist()
    return dict(zip(BLOCK_CLASSES, words))


def transform_sf(sb: torch.Tensor) -> torch.Tensor:
    l = lib()
    E, N, KB = sb.shape
    out = torch.empty(l.cdg_sf_atoms_bytes(E, N, KB), dtype=torch.uint8, device=sb.device)
    st = l.cdg_transform_sf(ctypes.c_void_p(sb.data_ptr()), sb.stride(0), sb.stride(1), E, N, KB,
                            ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == CDG_OK, st
    return out


def device_status(clear: bool = True) -> tuple[int, int]:
    """(status, first wait code) of cdg_device_status on the current device."""
    where = ctypes.c_int32(0)
    st = lib().cdg_device_status(1 if clear else 0, ctypes.byref(where))
    return st, where.value
