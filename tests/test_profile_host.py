"""CDG_PROFILE wrappers (consumer_deep_gemm/profile.py): the host-timed path on CPU, the
CUDA-event path on a GPU."""

import io
import types

import pytest

from consumer_deep_gemm import profile


def test_wrapped_functions_are_counted_and_reported():
    calls = []
    mod = types.SimpleNamespace(m_grouped_fp8_fp4_gemm_nt_contiguous=lambda *a, **k: calls.append(1) or 7,
                                transform_sf_into_required_layout=lambda x: x + 1)
    out = io.StringIO()
    prof = profile.install(mod, interval=3, out=out)
    for _ in range(4):
        assert mod.m_grouped_fp8_fp4_gemm_nt_contiguous(1, 2, recipe_a=(1, 128)) == 7
    assert mod.transform_sf_into_required_layout(1) == 2
    assert len(calls) == 4
    stats = prof.stats()
    assert stats["m_grouped_fp8_fp4_gemm_nt_contiguous"][0] == 4
    assert stats["transform_sf_into_required_layout"][0] == 1
    text = out.getvalue()
    assert "=== CDG Profile (3 calls) ===" in text and "m_grouped_fp8_fp4_gemm_nt_contiguous" in text
    assert "TOTAL" in text


@pytest.mark.gpu
def test_gpu_calls_are_timed_with_events():
    """On CUDA tensors the wrapper records events on the current stream; the resolved
    device times are positive and the wrapped GEMM still gives the unwrapped result."""
    import torch

    import consumer_deep_gemm as cdg
    from consumer_deep_gemm import synthetic

    inp = synthetic.make_inputs(synthetic.CONFIGS["c0"], device="cuda", seed=0)
    a, sa, b, sb, ids = inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"]
    mod = types.SimpleNamespace(m_grouped_fp8_fp4_gemm_nt_contiguous=cdg.m_grouped_fp8_fp4_gemm_nt_contiguous)
    prof = profile.install(mod, interval=1000)
    d1 = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device="cuda")
    d2 = torch.empty_like(d1)
    mod.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (b, sb), d1, ids)
    cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (b, sb), d2, ids)
    assert len(prof.pending) == 1
    calls, seconds = prof.stats()["m_grouped_fp8_fp4_gemm_nt_contiguous"]
    assert calls == 1 and seconds > 0
    assert torch.equal(d1.view(torch.int16), d2.view(torch.int16))
