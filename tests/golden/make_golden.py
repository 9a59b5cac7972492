"""Generate the golden fixtures from the reference implementation itself.

Run in the build container, where the reference checkout is importable::

    python tests/golden/make_golden.py --ref /path/to/Consumer-DeepGEMM   (or CDG_REFERENCE_ROOT=...)

The reference package is loaded under the alias ``ref_cdg`` (so it cannot clash
with this repository's ``consumer_deep_gemm``) and its CPU path is called on
seeded inputs:

* ``_m_grouped_fp8_fp4_fallback_nt``       (consumer_deep_gemm/gemm.py:343-367)
* ``_m_grouped_fp8_fp4_dequant_mm_nt``     (gemm.py:411-464)
* ``_reorder_scale_to_cutlass_sf_atom``    (gemm.py:76-116)
* ``_dequant_fp4_block``                   (gemm.py:147-187)
* ``_float_scale_to_e8m0``                 (gemm.py:62-73)
* ``m_grouped_fp8_fp4_gemm_nt_masked``     (gemm.py:529-551)
* ``transform_weights_for_mega_moe``       (mega.py:42-50)

``ue8m0x4_*`` cases hold activation scales that are powers of two, stored both as the
FP32 values the reference consumes and packed four UE8M0 bytes to an int32 word (the
format DeepGEMM's UE8M0 recipe passes; the reference itself only reads FP32 scales).

Cases cover the reference's own known answers (tests/test_fp4_fallback.py:15-73,
tests/test_native_abi.py:144-196, tests/test_scale_reorder.py:53-68,
tests/test_reorder_compare.py:8-35), benchmark config 0, and edge cases (empty
and ragged groups, interleaved and out-of-range ids, the psum form, BF16/FP32
activations, FP32 weight scales, K and N that are not tile multiples).
Tensors are stored as raw integer views (fp8 -> uint8, bf16 -> int16).
Nothing at test time reads the reference; the tests read these files only.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "consumer-deepgemm_b200"))


def load_reference(root: str):
    spec = importlib.util.spec_from_file_location(
        "ref_cdg", os.path.join(root, "consumer_deep_gemm", "__init__.py"),
        submodule_search_locations=[os.path.join(root, "consumer_deep_gemm")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_cdg"] = mod
    spec.loader.exec_module(mod)
    import ref_cdg.gemm as gemm  # noqa: E402
    return gemm


def raw(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()
    return t.numpy()


def gemm_case(gemm, name, a, sa, b, sb, m_indices, d_dtype=torch.bfloat16, fn="fallback"):
    m = a.shape[0]
    n = b.shape[1] if b.dim() == 3 else b.shape[0]
    d = torch.full((m, n), 7.0, dtype=d_dtype)  # non-zero: the op must overwrite every row
    a_arg = (a, sa) if sa is not None else a
    if fn == "fallback":
        gemm._m_grouped_fp8_fp4_fallback_nt(a_arg, (b, sb), d, m_indices)
    elif fn == "masked":
        gemm.m_grouped_fp8_fp4_gemm_nt_masked(a_arg, (b, sb), d, m_indices)
    else:
        gemm._m_grouped_fp8_fp4_dequant_mm_nt(a_arg, (b, sb), d, m_indices)
    out = {"a": raw(a), "a_dtype": str(a.dtype), "b": raw(b), "d": raw(d), "d_dtype": str(d_dtype)}
    if sa is not None:
        out["sa"] = raw(sa)
    out["sb"] = raw(sb)
    out["sb_dtype"] = str(sb.dtype)
    out["m_indices"] = raw(m_indices) if m_indices is not None else np.zeros(0, np.int32)
    out["has_m_indices"] = np.array(m_indices is not None)
    out["masked"] = np.array(fn == "masked")
    return name, out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CDG_REFERENCE_ROOT"),
                    help="checkout of the reference project (or set CDG_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or CDG_REFERENCE_ROOT")
    gemm = load_reference(args.ref)
    from consumer_deep_gemm import synthetic
    from deep_gemm.utils.math import per_block_cast_to_fp4, per_block_cast_to_fp8

    torch.manual_seed(0)
    cases = {}

    def add(item):
        cases[item[0]] = item[1]

    # --- known answers of the reference's own tests -------------------------------------
    packed = torch.tensor([[[0x21, 0x43]], [[0x44, 0x44]]], dtype=torch.uint8)
    sc = torch.full((2, 1, 1), 127, dtype=torch.uint8)
    ones4 = torch.ones((4, 4), dtype=torch.bfloat16)
    add(gemm_case(gemm, "kat_grouped_b", ones4, None, packed, sc, torch.tensor([0, 1, -1, 0], dtype=torch.int32)))
    add(gemm_case(gemm, "kat_interleaved", ones4, None, packed, sc, torch.tensor([1, 0, 1, 0], dtype=torch.int32)))
    a = torch.ones((128, 128), dtype=torch.float32).to(torch.float8_e4m3fn)
    add(gemm_case(gemm, "kat_all_128", a, torch.ones((128, 1)), torch.full((1, 128, 64), 0x22, dtype=torch.uint8),
                  torch.ones((1, 128, 4)), torch.zeros(128, dtype=torch.int32)))
    a = torch.ones((128, 256), dtype=torch.float32).to(torch.float8_e4m3fn)
    add(gemm_case(gemm, "kat_scale_1536", a, torch.tensor([[2.0, 4.0]] * 128),
                  torch.full((1, 128, 128), 0x22, dtype=torch.uint8), torch.full((1, 128, 8), 2.0),
                  torch.zeros(128, dtype=torch.int32)))
    mi = torch.full((256,), -1, dtype=torch.int32)
    mi[:17] = 0
    mi[128:151] = 1
    add(gemm_case(gemm, "kat_vllm_padding_zero", torch.zeros((256, 128), dtype=torch.float8_e4m3fn),
                  torch.ones((256, 1)), torch.zeros((2, 128, 64), dtype=torch.uint8), torch.ones((2, 128, 4)), mi))

    # --- benchmark config 0 (both reference paths) ----------------------------------------
    inp = synthetic.make_inputs(synthetic.CONFIGS["c0"], seed=0)
    name, c0 = gemm_case(gemm, "c0", inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"], fn="fallback")
    _, c0_mm = gemm_case(gemm, "c0", inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"], fn="dequant_mm")
    # The two reference paths agree bit for bit on per-row ids; keep one copy of the inputs.
    assert np.array_equal(c0["d"], c0_mm["d"])
    cases[name] = c0

    # --- edge cases -------------------------------------------------------------------------
    def rand_case(name, m, k, n, e, ids, a_kind="fp8", sb_kind="u8", d_dtype=torch.bfloat16, sa_cols=None, seed=1,
                  fn="fallback", single_b=False):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(m, k, generator=g)
        w = torch.randn(e, n, k, generator=g) * 0.02
        bq, sbq = per_block_cast_to_fp4(w)
        if sb_kind == "f32":
            sbq = torch.pow(2.0, sbq.float() - 127.0) * (1.0 + torch.rand(sbq.shape, generator=g))
        if a_kind == "fp8":
            cols = sa_cols or (k + 127) // 128
            aq, saq = per_block_cast_to_fp8(x, block_k=k // cols)
        elif a_kind == "bf16":
            aq, saq = x.to(torch.bfloat16), torch.ones(m, 1)
        else:
            aq, saq = x.float(), torch.ones(m, 1)
        if single_b:
            bq, sbq = bq[0], sbq[0]
        add(gemm_case(gemm, name, aq, saq, bq, sbq, ids, d_dtype=d_dtype, fn=fn))

    add_ids = lambda v: torch.tensor(v, dtype=torch.int32)  # noqa: E731
    rand_case("edge_empty", 256, 256, 128, 4, torch.full((256,), -1, dtype=torch.int32))
    ragged = torch.tensor([0] * 5 + [1] * 70 + [3] * 130 + [-1] * 51, dtype=torch.int32)
    rand_case("edge_ragged", 256, 256, 128, 4, ragged)
    inter = torch.randint(-1, 4, (256,), generator=torch.Generator().manual_seed(5)).to(torch.int32)
    rand_case("edge_interleaved", 256, 256, 128, 4, inter)
    oor = torch.tensor(([2] * 60 + [7] * 10 + [-3] * 10 + [1] * 48) * 2, dtype=torch.int32)
    rand_case("edge_out_of_range_ids", 256, 256, 128, 4, oor)
    rand_case("edge_psum", 384, 256, 128, 3, add_ids([100, 100, 300]))
    rand_case("edge_psum_int64", 384, 256, 128, 3, torch.tensor([128, 256, 384], dtype=torch.int64))
    rand_case("edge_bf16_a", 256, 256, 128, 2, add_ids([0] * 128 + [1] * 100 + [-1] * 28), a_kind="bf16")
    rand_case("edge_fp32_a", 256, 256, 128, 2, add_ids([1] * 128 + [0] * 128), a_kind="f32")
    rand_case("edge_fp32_sb", 256, 256, 128, 2, add_ids([0] * 128 + [1] * 128), sb_kind="f32")
    rand_case("edge_fp32_d", 256, 256, 128, 2, add_ids([0] * 100 + [-1] * 28 + [1] * 128), d_dtype=torch.float32)
    rand_case("edge_k192_blockk96", 128, 192, 48, 2, add_ids([1] * 64 + [0] * 64), sa_cols=2)
    rand_case("edge_n40_m200", 200, 128, 40, 3, torch.randint(0, 3, (200,), generator=torch.Generator().manual_seed(9)).to(torch.int32))
    rand_case("edge_aligned_3groups", 384, 512, 256, 3, add_ids([2] * 128 + [0] * 128 + [1] * 90 + [-1] * 38), seed=3)
    rand_case("edge_int64_ids", 256, 256, 128, 2, torch.tensor([1] * 128 + [0] * 128, dtype=torch.int64))
    # one block per size class: 20 rows (narrow), 30 rows (narrow), 7 rows (tiny), 100 rows (wide)
    sizes = torch.tensor(([1] * 20 + [-1] * 108) + ([0] * 30 + [-1] * 98) + ([2] * 7 + [-1] * 121)
                         + ([3] * 100 + [-1] * 28), dtype=torch.int32)
    rand_case("edge_block_classes", 512, 384, 256, 4, sizes, seed=8)

    # --- masked layout: G blocks of S = M // G rows, masked_m[g] leading rows each -----------
    rand_case("masked_aligned", 512, 256, 128, 4, add_ids([5, 128, 0, 77]), fn="masked", seed=11)
    rand_case("masked_s64", 384, 256, 256, 6, add_ids([1, 64, 33, 0, 16, 2]), fn="masked", seed=12)
    rand_case("masked_s160", 480, 256, 128, 3, add_ids([150, 3, 160]), fn="masked", seed=13)
    # counts above S run on into the next block (later groups win) and into the tail rows
    rand_case("masked_overspill", 305, 256, 128, 3, add_ids([130, 20, 110]), fn="masked", seed=14)
    rand_case("masked_int64_negative", 256, 256, 128, 4, torch.tensor([3, -5, 64, 0], dtype=torch.int64),
              fn="masked", seed=15)
    rand_case("masked_decode_classes", 2048, 512, 256, 8, add_ids([1, 16, 17, 32, 33, 128, 129, 256]), fn="masked",
              seed=16)
    rand_case("masked_single_b", 192, 256, 128, 1, add_ids([7]), fn="masked", single_b=True, seed=17)

    # --- power-of-two activation scales, also packed 4 UE8M0 bytes per int32 word ----------
    def packed_case(name, m, k, n, e, ids, seed):
        g = torch.Generator().manual_seed(seed)
        kb = (k + 127) // 128
        aq = (torch.randn(m, k, generator=g) * 64).to(torch.float8_e4m3fn)
        sbytes = torch.randint(112, 136, (m, kb), generator=g, dtype=torch.int32)
        sa_f32 = torch.pow(2.0, sbytes.float() - 127.0)
        w = torch.randn(e, n, k, generator=g) * 0.02
        bq, sbq = per_block_cast_to_fp4(w)
        words = (kb + 3) // 4
        padded = torch.full((m, words * 4), 127, dtype=torch.int32)
        padded[:, :kb] = sbytes
        packed = (padded[:, 0::4] | (padded[:, 1::4] << 8) | (padded[:, 2::4] << 16) | (padded[:, 3::4] << 24))
        name, case = gemm_case(gemm, name, aq, sa_f32, bq, sbq, ids)
        case["sa_packed"] = packed.to(torch.int32).numpy()
        cases[name] = case

    packed_case("ue8m0x4_ragged", 512, 512, 256, 4,
                add_ids([0] * 100 + [-1] * 28 + [2] * 128 + [1] * 3 + [-1] * 125 + [3] * 128), seed=21)
    packed_case("ue8m0x4_k1024", 256, 1024, 256, 2, add_ids([1] * 200 + [-1] * 56), seed=22)
    packed_case("ue8m0x4_k640_n128", 256, 640, 128, 2, add_ids([0] * 128 + [1] * 64 + [-1] * 64), seed=23)

    # --- byte-level helpers -----------------------------------------------------------------
    sf = torch.arange(128 * 8, dtype=torch.uint8).reshape(128, 8)
    cases["sf_reorder_arange"] = {"src": raw(sf), "dst": raw(gemm._reorder_scale_to_cutlass_sf_atom(sf, 128, 8))}
    sf = torch.randint(0, 256, (300, 10), dtype=torch.uint8, generator=torch.Generator().manual_seed(4))
    cases["sf_reorder_padded"] = {"src": raw(sf), "dst": raw(gemm._reorder_scale_to_cutlass_sf_atom(sf, 300, 10))}
    allb = torch.arange(256, dtype=torch.uint8).repeat(4, 16).reshape(4, 16, 256)
    scl = torch.randint(100, 150, (4, 16, 16), dtype=torch.uint8, generator=torch.Generator().manual_seed(6))
    cases["fp4_dequant_all_bytes"] = {"src": raw(allb), "scale": raw(scl), "dst": raw(gemm._dequant_fp4_block(allb, scl))}
    # MegaMoE weight layout (mega.py:42-50): L1 N=256 (gate|up), L2 N=128, plus an L2 whose
    # row count is not a multiple of 128 (scales returned unchanged)
    import ref_cdg.mega as ref_mega
    gm = torch.Generator().manual_seed(31)
    mk = lambda *shape: torch.randint(0, 256, shape, dtype=torch.uint8, generator=gm)  # noqa: E731
    w1, s1, w2, s2 = mk(2, 256, 64), mk(2, 256, 8), mk(2, 128, 32), mk(2, 128, 4)
    (ow1, os1), (ow2, os2) = ref_mega.transform_weights_for_mega_moe((w1, s1), (w2, s2))
    w2b, s2b = mk(3, 96, 16), mk(3, 96, 2)
    (_, _), (ow2b, os2b) = ref_mega.transform_weights_for_mega_moe((w1, s1), (w2b, s2b))
    cases["mega_moe_transform"] = {
        "w1": raw(w1), "s1": raw(s1), "w2": raw(w2), "s2": raw(s2), "w2b": raw(w2b), "s2b": raw(s2b),
        "ow1": raw(ow1), "os1": raw(os1), "ow2": raw(ow2), "os2": raw(os2), "ow2b": raw(ow2b), "os2b": raw(os2b)}
    fs = torch.tensor([1.0, 2.0, 0.75, 3.0, 1e-30, 1e30, 0.0, 5.9e-39, 1.5, 2.9999])
    cases["float_scale_to_e8m0"] = {"src": raw(fs), "dst": raw(gemm._float_scale_to_e8m0(fs))}

    for name, arrays in cases.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(f"wrote {len(cases)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
