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
