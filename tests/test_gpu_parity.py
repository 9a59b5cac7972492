"""GPU parity of the grouped FP8 x MXFP4 GEMM, driven through the C ABI (ctypes).

Every golden case (outputs of the reference itself, see tests/golden/make_golden.py)
is run three times: through the default dispatch (tensor-core kernels where the
inputs fit them -- CTA pairs when N is a multiple of 256 -- and the exact SIMT
kernel for the rest), with single-CTA tensor-core kernels, and with the SIMT
kernel forced.

Tolerances, against the reference's BF16 output over the routed rows:
  * max |out - ref| / max |ref|      <= 1e-2   (TOL_NORMWISE)
  * per-row ||out - ref|| / ||ref||  <= 2e-3   (TOL_ROW_L2)
  * rows without a valid group id are exactly zero, bit for bit;
  * known-answer cases (small integers) are exact.
At the benchmark sizes (configs c1-c3, and c2u/c3u with power-of-two activation
scales) every routed row is checked against the oracle run on the GPU's own FP32
arithmetic (TF32 off), expert by expert, with the same tolerances, plus
bit-identical repeat runs and exact zero rows.
"""

import pytest
import torch

import cabi
from conftest import GEMM_CASES, MASKED_CASES, PACKED_SCALE_CASES, load_gemm_case
from metrics import TOL_NORMWISE, TOL_ROW_L2, errors
from oracle import cdg_oracle as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _invalid_rows(c) -> torch.Tensor:
    m = c["a"].shape[0]
    ids = c["m_indices"]
    e = c["b"].shape[0]
    if ids is None:
        return torch.zeros(m, dtype=torch.bool)
    ids = ids.to(torch.int64)
    if ids.numel() == m:
        return (ids < 0) | (ids >= e)
    covered = torch.zeros(m, dtype=torch.bool)
    start = 0
    for end in ids.tolist():
        covered[start:max(start, min(end, m))] = True
        start = end
    return ~covered


def _run_case(c, flags):
    a = c["a"].to(DEV)
    sa = c["sa"].to(DEV).float() if (c["sa"] is not None and a.dtype == torch.float8_e4m3fn) else None
    if a.dtype == torch.float8_e4m3fn and sa is None:
        sa = torch.ones(a.shape[0], (a.shape[1] + 127) // 128, device=DEV)
    b = c["b"].to(DEV)
    sb = c["sb"].to(DEV)
    ids = c["m_indices"].to(DEV) if c["m_indices"] is not None else None
    d = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    cabi.gemm(a, sa, b, sb, d, ids, flags=flags)
    torch.cuda.synchronize()
    return d.cpu()


@pytest.mark.parametrize("flags", [0, cabi.FLAG_SINGLE_CTA, cabi.FLAG_FORCE_GENERIC],
                         ids=["dispatch", "single_cta", "simt"])
@pytest.mark.parametrize("name", GEMM_CASES)
def test_golden_case(name, flags):
    c = load_gemm_case(name)
    out = _run_case(c, flags)
    ref = c["d"]
    assert not torch.isnan(out).any(), "rows left unwritten"
    bad = _invalid_rows(c)
    if bool(bad.any()):
        assert bool((out[bad].float() == 0).all()) and bool((torch.signbit(out[bad].float()) == 0).all())
    if name.startswith("kat_"):
        assert torch.equal(out, ref)
        return
    nw, rl2 = errors(out, ref, ~bad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (name, nw, rl2)


def _row_table(m, n, skip_every, seed):
    """A destination buffer [m + 3, n] of NaNs and a row table that stores GEMM row r at
    destination row perm[r] (a seeded permutation), except every `skip_every`-th row
    (address 0: not stored)."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(m + 3, generator=g)[:m]
    dst = torch.full((m + 3, n), float("nan"), dtype=torch.bfloat16, device=DEV)
    addr = dst.data_ptr() + perm.to(torch.int64) * (n * 2)
    skipped = torch.zeros(m, dtype=torch.bool)
    if skip_every:
        skipped[::skip_every] = True
    addr[skipped] = 0
    return dst, addr.to(DEV), perm, skipped


@pytest.mark.parametrize("flags", [0, cabi.FLAG_SINGLE_CTA, cabi.FLAG_FORCE_GENERIC],
                         ids=["dispatch", "single_cta", "simt"])
@pytest.mark.parametrize("name", ["c0", "edge_block_classes", "kat_vllm_padding_zero", "pow2_c0"])
def test_row_table_output_equals_plain_output(name, flags):
    """D through a row table (cdg_gemm_args.d_rows, how the expert-parallel layer returns FC2
    rows straight into the source ranks' windows): every stored row is bit-identical to the
    same call's plain output (padding rows included, as zeros); rows whose address is 0 are
    not written; `d` itself is not read or written (NULL).  pow2_c0: c0 with power-of-two
    activation scales, so the direct class runs too."""
    c = load_gemm_case(name[5:] if name.startswith("pow2_") else name)
    if name.startswith("pow2_"):
        c = dict(c, sa=_pow2_scales(c["sa"]))
    plain = _run_case(c, flags)
    a = c["a"].to(DEV)
    sa = c["sa"].to(DEV).float()
    b, sb = c["b"].to(DEV), c["sb"].to(DEV)
    ids = c["m_indices"].to(DEV) if c["m_indices"] is not None else None
    m, n = plain.shape
    dst, addr, perm, skipped = _row_table(m, n, 5, seed=11)
    shape_only = torch.empty(1, n, dtype=torch.bfloat16, device=DEV).expand(m, n)
    cabi.gemm(a, sa, b, sb, shape_only, ids, flags=flags, d_rows=addr)
    torch.cuda.synchronize()
    out = dst.cpu()
    kept = ~skipped
    assert torch.equal(out[perm[kept]].view(torch.int16), plain[kept].view(torch.int16))
    untouched = torch.ones(m + 3, dtype=torch.bool)
    untouched[perm[kept]] = False
    assert bool(torch.isnan(out[untouched].float()).all())
    assert cabi.device_status() == (0, 0)


def test_row_table_misaligned_address_is_skipped_and_reported():
    """A D row address that is not 16-byte aligned: that row is not written, the call's other
    rows are, and the device record reports CDG_ERR_DEVICE_INDEX (9).  Every kernel checks the
    address before its store, so nothing faults."""
    c = load_gemm_case("c0")
    a, sa = c["a"].to(DEV), c["sa"].to(DEV).float()
    b, sb, ids = c["b"].to(DEV), c["sb"].to(DEV), c["m_indices"].to(DEV)
    plain = _run_case(c, 0)
    m, n = plain.shape
    dst, addr, perm, skipped = _row_table(m, n, 0, seed=12)
    routed = (c["m_indices"] >= 0).nonzero().flatten()
    bad = int(routed[0])
    addr[bad] += 2  # inside the row's own bytes, but not 16-byte aligned
    shape_only = torch.empty(1, n, dtype=torch.bfloat16, device=DEV).expand(m, n)
    cabi.gemm(a, sa, b, sb, shape_only, ids, d_rows=addr, check_status=False)
    torch.cuda.synchronize()
    out = dst.cpu()
    assert bool(torch.isnan(out[perm[bad]].float()).all())
    keep = torch.ones(m, dtype=torch.bool)
    keep[bad] = False
    assert torch.equal(out[perm[keep]].view(torch.int16), plain[keep].view(torch.int16))
    st, _ = cabi.device_status()
    assert st == 9
    assert cabi.device_status() == (0, 0)


def _masked_covered(m, counts, groups):
    """Rows the masked layout writes from a group (the rest must be zero)."""
    covered = torch.zeros(m, dtype=torch.bool)
    block = m // groups
    for g, cnt in enumerate(counts.tolist()):
        if cnt > 0:
            covered[g * block:min(m, g * block + cnt)] = True
    return covered


@pytest.mark.parametrize("flags", [0, cabi.FLAG_SINGLE_CTA, cabi.FLAG_FORCE_GENERIC],
                         ids=["dispatch", "single_cta", "simt"])
@pytest.mark.parametrize("name", MASKED_CASES)
def test_masked_golden_case(name, flags):
    """Masked layout through cdg_grouped_fp8_fp4_gemm_nt_masked against the reference."""
    c = load_gemm_case(name)
    a = c["a"].to(DEV)
    sa = c["sa"].to(DEV).float()
    b, sb = c["b"].to(DEV), c["sb"].to(DEV)
    single = b.dim() == 2
    if single:
        b, sb = b.unsqueeze(0), sb.unsqueeze(0)
    d = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    ids = None if single else c["m_indices"].to(DEV)
    cabi.gemm(a, sa, b, sb, d, ids, flags=flags, masked=True)
    torch.cuda.synchronize()
    out, ref = d.cpu(), c["d"]
    assert not torch.isnan(out).any(), "rows left unwritten"
    rows = torch.ones(a.shape[0], dtype=torch.bool) if single else _masked_covered(a.shape[0], c["m_indices"],
                                                                                   b.shape[0])
    if bool((~rows).any()):
        assert bool((out[~rows].float() == 0).all())
    nw, rl2 = errors(out, ref, rows)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (name, nw, rl2)


@pytest.mark.parametrize("mn_major", [False, True], ids=["row_major", "mn_major"])
@pytest.mark.parametrize("flags", [0, cabi.FLAG_SINGLE_CTA, cabi.FLAG_FORCE_GENERIC],
                         ids=["dispatch", "single_cta", "simt"])
@pytest.mark.parametrize("name", PACKED_SCALE_CASES)
def test_packed_ue8m0_activation_scales(name, flags, mn_major):
    """int32 words of 4 UE8M0 scales (row-major, or MN-major as DeepGEMM lays them out)."""
    c = load_gemm_case(name)
    a = c["a"].to(DEV)
    words = c["sa_packed"].to(DEV)
    if mn_major:  # [words, M_aligned] storage viewed as [M, words]
        m = words.shape[0]
        store = torch.zeros(words.shape[1], (m + 3) // 4 * 4, dtype=torch.int32, device=DEV)
        store[:, :m] = words.t()
        words = store.t()[:m]
    b, sb = c["b"].to(DEV), c["sb"].to(DEV)
    ids = c["m_indices"].to(DEV)
    d = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    cabi.gemm(a, words, b, sb, d, ids, flags=flags)
    torch.cuda.synchronize()
    out = d.cpu()
    bad = _invalid_rows(c)
    assert not torch.isnan(out).any()
    assert bool((out[bad].float() == 0).all())
    nw, rl2 = errors(out, c["d"], ~bad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (name, nw, rl2)


def _pow2_scales(sa: torch.Tensor) -> torch.Tensor:
    """FP32 activation scales rounded up to powers of two (as UE8M0 quantisation recipes do)."""
    return torch.exp2(torch.ceil(torch.log2(sa.float().clamp(min=2.0 ** -100))))


POW2_CASES = [n for n in GEMM_CASES + MASKED_CASES + PACKED_SCALE_CASES
              if n.startswith(("c0", "edge_block_classes", "edge_ragged", "edge_interleaved", "edge_aligned",
                               "edge_psum", "edge_n40", "edge_int64", "masked_", "ue8m0x4_"))]


@pytest.mark.parametrize("flags", [0, cabi.FLAG_SINGLE_CTA], ids=["dispatch", "single_cta"])
@pytest.mark.parametrize("name", POW2_CASES)
def test_power_of_two_fp32_scales(name, flags):
    """FP32 activation scales that are all powers of two: wide blocks take the direct class
    (raw e4m3 rows, scales as UE8M0 MMA scale factors) on the CTA-pair path.  Checked
    against the oracle on the same inputs, same tolerances as the golden cases."""
    c = load_gemm_case(name)
    if c["a"].dtype != torch.float8_e4m3fn or c["sa"] is None:
        pytest.skip("activation scales only apply to FP8 activations")
    sa = _pow2_scales(c["sa"])
    masked = c["masked"] or name.startswith("masked_")
    b, sb = c["b"], c["sb"]
    if masked and b.dim() == 2:
        b, sb = b.unsqueeze(0), sb.unsqueeze(0)
    ids = c["m_indices"]
    if masked and c["b"].dim() == 2:
        ids = None
    ref = torch.empty(c["d"].shape, dtype=c["d_dtype"])
    if masked:
        oracle.m_grouped_fp8_fp4_gemm_nt_masked((c["a"], sa), (c["b"], c["sb"]), ref, ids)
    else:
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((c["a"], sa), (b, sb), ref, ids)
    d = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    ws = cabi.gemm(c["a"].to(DEV), sa.to(DEV), b.to(DEV), sb.to(DEV), d, None if ids is None else ids.to(DEV),
                   flags=flags, masked=masked)
    torch.cuda.synchronize()
    out = d.cpu()
    assert not torch.isnan(out).any(), "rows left unwritten"
    if masked:
        rows = (torch.ones(out.shape[0], dtype=torch.bool) if ids is None
                else _masked_covered(out.shape[0], ids, b.shape[0]))
    else:
        rows = ~_invalid_rows(c)
    assert bool((out[~rows].float() == 0).all())
    nw, rl2 = errors(out, ref, rows)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (name, nw, rl2)
    cls = cabi.block_classes(ws)
    if flags == 0 and b.shape[1] % 256 == 0:
        assert cls["wide"] == 0, cls  # every wide block had power-of-two scales
    else:
        assert cls["wide_direct"] == 0, cls  # the direct class is a CTA-pair kernel


def test_direct_class_is_per_block():
    """One scale that is not a power of two keeps its block on the two-plane path while
    the other wide blocks go direct; both kinds of block match the oracle."""
    c = load_gemm_case("ue8m0x4_ragged")
    sa = c["sa"].float().clone()
    ids = c["m_indices"]
    e0_rows = (ids == int(ids[ids >= 0][0])).nonzero().flatten()
    sa[int(e0_rows[3]), 1] *= 1.5
    ref = torch.empty(c["d"].shape, dtype=c["d_dtype"])
    oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((c["a"], sa), (c["b"], c["sb"]), ref, ids)
    d = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    ws = cabi.gemm(c["a"].to(DEV), sa.to(DEV), c["b"].to(DEV), c["sb"].to(DEV), d, ids.to(DEV))
    torch.cuda.synchronize()
    cls = cabi.block_classes(ws)
    assert cls["wide"] >= 1 and cls["wide_direct"] >= 1, cls
    bad = _invalid_rows(c)
    out = d.cpu()
    assert bool((out[bad].float() == 0).all())
    nw, rl2 = errors(out, ref, ~bad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (nw, rl2)


def test_exponent_outside_scale_factor_range_goes_to_simt():
    """A wide block whose row exponent 2^E is below UE8M0's range (denormal FP32 scales) is
    planned for the exact SIMT kernel; its rows match a forced-SIMT run bit for bit, and the
    other blocks still match the oracle."""
    c = load_gemm_case("c0")
    sa = c["sa"].float().clone()
    ids = c["m_indices"]
    blk = 3  # a block of one expert with more than 32 routed rows
    rows = torch.arange(blk * 128, blk * 128 + 128)
    assert int((ids[rows] >= 0).sum()) > 32
    sa[rows] *= 2.0 ** -124  # BF16 denormal scales: E near -130
    a, b, sb = c["a"].to(DEV), c["b"].to(DEV), c["sb"].to(DEV)
    d = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    ws = cabi.gemm(a, sa.to(DEV), b, sb, d, ids.to(DEV))
    torch.cuda.synchronize()
    assert cabi.block_classes(ws)["irregular"] >= 1
    d_simt = torch.full(c["d"].shape, float("nan"), dtype=c["d_dtype"], device=DEV)
    cabi.gemm(a, sa.to(DEV), b, sb, d_simt, ids.to(DEV), flags=cabi.FLAG_FORCE_GENERIC)
    torch.cuda.synchronize()
    out, out_simt = d.cpu(), d_simt.cpu()
    assert torch.equal(out[rows].view(torch.int16), out_simt[rows].view(torch.int16))
    ref = torch.empty(c["d"].shape, dtype=c["d_dtype"])
    oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((c["a"], sa), (c["b"], c["sb"]), ref, ids)
    keep = ~_invalid_rows(c)
    keep[rows] = False
    nw, rl2 = errors(out, ref, keep)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (nw, rl2)


def test_packed_scales_public_api():
    import consumer_deep_gemm as cdg

    c = load_gemm_case("ue8m0x4_ragged")
    d = torch.empty(c["d"].shape, dtype=torch.bfloat16, device=DEV)
    cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((c["a"].to(DEV), c["sa_packed"].to(DEV)), (c["b"].to(DEV), c["sb"].to(DEV)),
                                             d, c["m_indices"].to(DEV), recipe_a=(1, 128), recipe_b=(1, 32))
    torch.cuda.synchronize()
    bad = _invalid_rows(c)
    nw, rl2 = errors(d.cpu(), c["d"], ~bad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (nw, rl2)


def test_masked_public_api_3d_views():
    """[G, S, K] activations and [G, S, N] output through the Python entry, masked_m on the host."""
    import consumer_deep_gemm as cdg
    from metrics import errors as _errors

    c = load_gemm_case("masked_decode_classes")
    G = c["b"].shape[0]
    a3 = c["a"].view(G, -1, c["a"].shape[1]).to(DEV)
    sa3 = c["sa"].float().view(G, -1, c["sa"].shape[1]).to(DEV)
    d3 = torch.full((G, a3.shape[1], c["d"].shape[1]), float("nan"), dtype=torch.bfloat16, device=DEV)
    cdg.m_grouped_fp8_fp4_gemm_nt_masked((a3, sa3), (c["b"].to(DEV), c["sb"].to(DEV)), d3, c["m_indices"],
                                         expected_m=64)
    torch.cuda.synchronize()
    out = d3.view(-1, d3.shape[2]).cpu()
    rows = _masked_covered(out.shape[0], c["m_indices"], G)
    assert bool((out[~rows].float() == 0).all())
    nw, rl2 = _errors(out, c["d"], rows)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (nw, rl2)


def test_sf_transform_bit_exact_vs_oracle():
    g = torch.Generator().manual_seed(3)
    for e, n, kb in [(3, 256, 16), (2, 384, 128), (1, 128, 4)]:
        sb = torch.randint(0, 256, (e, n, kb), dtype=torch.uint8, generator=g)
        out = cabi.transform_sf(sb.to(DEV)).cpu().numpy()
        ref = [oracle.reorder_scale_to_sf_atom(sb[i].numpy()) for i in range(e)]
        import numpy as np
        assert np.array_equal(out, np.concatenate(ref)), (e, n, kb)


def test_atoms_and_row_major_scales_agree():
    """The GEMM given pre-transformed scale atoms equals the GEMM given row-major scales, bit for bit."""
    c = load_gemm_case("c0")
    a, sa = c["a"].to(DEV), c["sa"].to(DEV)
    b, sb, ids = c["b"].to(DEV), c["sb"].to(DEV), c["m_indices"].to(DEV)
    d1 = torch.empty(c["d"].shape, dtype=torch.bfloat16, device=DEV)
    d2 = torch.empty_like(d1)
    cabi.gemm(a, sa, b, sb, d1, ids)
    atoms = cabi.transform_sf(sb)
    cabi.gemm(a, sa, b, atoms, d2, ids, sb_atoms=True)
    torch.cuda.synchronize()
    assert torch.equal(d1.view(torch.int16), d2.view(torch.int16))


def test_padding_rows_with_garbage_do_not_leak():
    """vLLM reuses workspaces: padding rows of A can hold any bytes (NaN included)."""
    c = load_gemm_case("c0")
    a = c["a"].clone()
    ids = c["m_indices"]
    pad = ids < 0
    g = torch.Generator().manual_seed(11)
    a.view(torch.uint8)[pad] = torch.randint(0, 256, (int(pad.sum()), a.shape[1]), dtype=torch.uint8, generator=g)
    sa = c["sa"].clone()
    sa[pad] = float("nan")
    c2 = dict(c, a=a, sa=sa)
    out = _run_case(c2, 0)
    assert bool((out[pad].float() == 0).all())
    nw, rl2 = errors(out, c["d"], ~pad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2


def _full_oracle_on_device(inp) -> torch.Tensor:
    """The oracle's D for every row, computed with the operands where they lie (the GPU).

    The oracle is pure torch; run on CUDA tensors its per-group FP32 products are cuBLAS
    FP32 GEMMs (TF32 switched off here), its dequantisation the same BF16 roundings.
    """
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a, sa, b, sb, ids = inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"]
        ref = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=a.device)
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (b, sb), ref, ids)
        return ref
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3", "c2u", "c3u"])
def test_benchmark_config_every_row(cfg):
    from consumer_deep_gemm import synthetic

    inp = synthetic.make_inputs(synthetic.CONFIGS[cfg], device=DEV, seed=0)
    a, sa, b, sb, ids = inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"]
    m, n = a.shape[0], b.shape[1]
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV)
    ws = cabi.gemm(a, sa, b, sb, d, ids)
    classes = cabi.block_classes(ws)
    d2 = torch.empty_like(d)
    cabi.gemm(a, sa, b, sb, d2, ids)
    torch.cuda.synchronize()
    assert torch.equal(d.view(torch.int16), d2.view(torch.int16)), "repeat run differs"
    del d2
    pad = ids < 0
    assert bool((d[pad] == 0).all()), "padding rows must be zero"
    assert not bool(torch.isnan(d).any())
    ref = _full_oracle_on_device(inp)
    valid = ~pad
    nw, rl2 = errors(d[valid], ref[valid])
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (cfg, classes, nw, rl2)
    # the single-CTA kernels (same tiles, one SM each) agree on every row as well
    d1 = torch.full_like(d, float("nan"))
    cabi.gemm(a, sa, b, sb, d1, ids, flags=cabi.FLAG_SINGLE_CTA)
    torch.cuda.synchronize()
    assert bool((d1[pad] == 0).all()) and not bool(torch.isnan(d1).any())
    nw1, rl21 = errors(d1[valid], ref[valid])
    assert nw1 <= TOL_NORMWISE and rl21 <= TOL_ROW_L2, (cfg, "single CTA", nw1, rl21)
    assert cabi.device_status() == (0, 0)


def _c0_on_device():
    c = load_gemm_case("c0")
    return [c[k].to(DEV) for k in ("a", "sa", "b", "sb", "m_indices")]


def test_float_weight_scales_that_are_powers_of_two_run_on_the_tensor_cores():
    """FP32 weight scales holding powers of two (2^(s-127) of the UE8M0 bytes): converted on the
    device to the same codes, every block on the tensor-core kernels, output bit-identical to
    the UE8M0 call; the weight-load hook turns them into the same atoms as the bytes."""
    import consumer_deep_gemm as cdg

    a, sa, b, sb, ids = _c0_on_device()
    sbf = torch.exp2(sb.float() - 127.0)
    d_u8 = torch.full((a.shape[0], b.shape[1]), float("nan"), dtype=torch.bfloat16, device=DEV)
    d_f = torch.full_like(d_u8, float("nan"))
    cabi.gemm(a, sa, b, sb, d_u8, ids)
    ws = cabi.gemm(a, sa, b, sbf, d_f, ids)
    classes = cabi.block_classes(ws)
    torch.cuda.synchronize()
    assert classes["irregular"] == 0 and classes["tiny"] + classes["narrow"] + classes["wide"] > 0, classes
    assert torch.equal(d_f.view(torch.int16), d_u8.view(torch.int16))
    assert torch.equal(cdg.transform_sf_into_required_layout(sbf), cdg.transform_sf_into_required_layout(sb))


def test_float_weight_scales_otherwise_stay_exact_on_the_simt_kernel():
    """FP32 weight scales that are not all powers of two: the device sends every block to the
    exact SIMT kernel (the reference's dequant fallback), matching the reference's output."""
    c = load_gemm_case("edge_fp32_sb")
    a, sa, b, sb, ids = (c[k].to(DEV) for k in ("a", "sa", "b", "sb", "m_indices"))
    assert sb.dtype == torch.float32
    d = torch.full(c["d"].shape, float("nan"), dtype=torch.bfloat16, device=DEV)
    ws = cabi.gemm(a, sa, b, sb, d, ids)
    classes = cabi.block_classes(ws)
    torch.cuda.synchronize()
    assert classes["tiny"] + classes["narrow"] + classes["wide"] + classes["wide_direct"] == 0, classes
    bad = _invalid_rows(c)
    nw, rl2 = errors(d.cpu(), c["d"], ~bad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2


def test_round_weight_scales_flag_uses_the_references_rounding():
    """CDG_FLAG_ROUND_SFB: float weight scales rounded to the nearest power of two on the device
    give the same bits as the UE8M0 call on the oracle's _float_scale_to_e8m0 codes (pinned to
    the reference's own outputs)."""
    a, sa, b, sb, ids = _c0_on_device()
    g = torch.Generator().manual_seed(21)
    sbf = (torch.exp2(sb.float() - 127.0).cpu() * (0.75 + 0.7 * torch.rand(sb.shape, generator=g))).to(DEV)
    codes = oracle.float_scale_to_e8m0(sbf.cpu()).to(DEV)
    d_r = torch.full((a.shape[0], b.shape[1]), float("nan"), dtype=torch.bfloat16, device=DEV)
    d_c = torch.full_like(d_r, float("nan"))
    cabi.gemm(a, sa, b, sbf, d_r, ids, flags=cabi.FLAG_ROUND_SFB)
    cabi.gemm(a, sa, b, codes, d_c, ids)
    torch.cuda.synchronize()
    assert torch.equal(d_r.view(torch.int16), d_c.view(torch.int16))


def _torch_planes(a, sa):
    """The two e4m3 activation planes and row exponents the GEMM forms from e4m3 rows with FP32
    1x128 scales: x = bf16(bf16(a) * bf16(s)), E = frexp exponent of the row's largest |bf16(s)|,
    hi = e4m3(x / 2^E), lo = e4m3(x / 2^E - hi)."""
    m, k = a.shape
    sb = sa.to(torch.bfloat16)
    x = (a.to(torch.bfloat16).view(m, k // 128, 128) * sb.unsqueeze(-1)).view(m, k)
    smax = sb.float().abs().nan_to_num(0.0, 0.0, 0.0).amax(dim=1)
    e = torch.where(smax > 0, torch.frexp(smax).exponent, torch.zeros_like(smax, dtype=torch.int32))
    v = x.float() * torch.exp2(-e.float()).unsqueeze(1)
    hi = v.to(torch.float8_e4m3fn)
    lo = (v - hi.float()).to(torch.float8_e4m3fn)
    return torch.stack([hi.view(torch.uint8), lo.view(torch.uint8)]).contiguous(), e.to(torch.int32).contiguous()


@pytest.mark.parametrize("name", ["c0", "edge_block_classes", "kat_vllm_padding_zero"])
def test_planes_form_equals_rows_form(name):
    """CDG_DTYPE_E4M3_PLANES: the GEMM on activation planes made outside it (as the MoE layer's
    quantising steps make them) gives the bits of the call on the e4m3 rows and scales."""
    from consumer_deep_gemm import native

    c = load_gemm_case(name)
    if c["a"].dtype != torch.float8_e4m3fn or c["a"].shape[0] % 128 or c["b"].shape[1] % 128 or \
            c["a"].shape[1] % 128 or c["sb"].dtype != torch.uint8 or c["m_indices"] is None or \
            c["m_indices"].numel() != c["a"].shape[0]:
        pytest.skip("outside the planes form's envelope")
    a, sa, b, sb, ids = (c[k].to(DEV) for k in ("a", "sa", "b", "sb", "m_indices"))
    d_rows = torch.full((a.shape[0], b.shape[1]), float("nan"), dtype=torch.bfloat16, device=DEV)
    cabi.gemm(a, sa.float(), b, sb, d_rows, ids)
    planes, rexp = _torch_planes(a, sa.float())
    d_pl = torch.full_like(d_rows, float("nan"))
    native.require().grouped_gemm_planes(planes, rexp, b, sb, d_pl, ids.to(torch.int32).contiguous(), 0)
    torch.cuda.synchronize()
    assert torch.equal(d_pl.view(torch.int16), d_rows.view(torch.int16))
    assert cabi.device_status() == (0, 0)


def test_mega_moe_transform_bytes_match_reference():
    import numpy as np

    import consumer_deep_gemm as cdg
    from conftest import GOLDEN

    z = np.load(f"{GOLDEN}/mega_moe_transform.npz")
    t = lambda k: torch.from_numpy(z[k]).to(DEV)  # noqa: E731
    (w1, s1), (w2, s2) = cdg.transform_weights_for_mega_moe((t("w1"), t("s1")), (t("w2"), t("s2")))
    for got, key in ((w1, "ow1"), (s1, "os1"), (w2, "ow2"), (s2, "os2")):
        assert np.array_equal(got.cpu().numpy(), z[key]), key
    _, (w2b, s2b) = cdg.transform_weights_for_mega_moe((t("w1"), t("s1")), (t("w2b"), t("s2b")))
    assert np.array_equal(w2b.cpu().numpy(), z["ow2b"]) and np.array_equal(s2b.cpu().numpy(), z["os2b"])
    # strided views (a weight slice of a larger tensor) take the same path
    big = torch.zeros(2, 256, 80, dtype=torch.uint8, device=DEV)
    big[:, :, :64] = t("w1")
    (w1v, _), _ = cdg.transform_weights_for_mega_moe((big[:, :, :64], t("s1")), (t("w2"), t("s2")))
    assert np.array_equal(w1v.cpu().numpy(), z["ow1"])
    with pytest.raises(NotImplementedError):
        cdg.fp8_fp4_mega_moe(None, None, None, None)
