"""bench.py's float32 layer reference (the checker behind the bench line's `parity` key) agrees
with the CPU reference layer of the tests (moe_ref.TorchRefOps over the oracle GEMM): the same
quantisation, dequantisation and roundings, so the outputs are equal up to FP32 summation order
(per-row relative L2 <= 1e-3; both recipes of activation scales)."""

import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402
from metrics import errors  # noqa: E402
from moe_ref import TorchRefOps, cast_to_fp8_pow2, make_layer_inputs  # noqa: E402


@pytest.mark.parametrize("ue8m0", [False, True], ids=["fp32", "ue8m0"])
def test_bench_layer_reference_matches_cpu_reference_layer(ue8m0):
    from consumer_deep_gemm.moe import MoELayer

    cfg = dict(tokens=24, experts=8, hidden=256, inter=128, topk=2)
    x, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**cfg)
    y_ref = MoELayer(w1, w1s, w2, w2s, num_experts=cfg["experts"], ops=TorchRefOps(), ue8m0=ue8m0)(x, ids, w)
    y = bench.layer_reference(x, ids.long(), w, w1, w1s, w2, w2s, ue8m0=ue8m0)
    nw, rl2 = errors(y, y_ref)
    assert nw <= 1e-3 and rl2 <= 1e-3, (nw, rl2)


def test_bench_pow2_quantiser_matches_the_tests_one():
    g = torch.Generator().manual_seed(4)
    x = torch.randn(16, 512, generator=g) * 3
    q1, s1 = bench._quant_pow2(x)
    q2, s2 = cast_to_fp8_pow2(x)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2)


def test_bench_cpu_impl_matches_the_oracle():
    """The CPU implementation the bench times (the reference's own pure-torch path from
    baseline/_ref when that install exists, else the oracle) gives the oracle's bits on a
    golden case, so the timed CPU baseline computes what the parity tests check against."""
    from conftest import load_gemm_case
    from oracle import cdg_oracle as oracle

    impl = bench.cpu_impl()
    c = load_gemm_case("edge_aligned_3groups")
    d = torch.empty(c["d"].shape, dtype=torch.bfloat16)
    impl["gemm"]((c["a"], c["sa"]), (c["b"], c["sb"]), d, c["m_indices"])
    d_or = torch.empty_like(d)
    oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((c["a"], c["sa"]), (c["b"], c["sb"]), d_or, c["m_indices"])
    assert torch.equal(d.view(torch.int16), d_or.view(torch.int16)), impl["kind"]
    g = torch.Generator().manual_seed(5)
    x = torch.randn(8, 384, generator=g) * 2
    from deep_gemm.utils.math import per_block_cast_to_fp8

    q1, s1 = impl["quant"](x)
    q2, s2 = per_block_cast_to_fp8(x)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2)
