"""Pins the CPU oracle to the reference: every golden fixture must be reproduced bit for bit."""

import os

import numpy as np
import torch

import pytest

from conftest import GOLDEN, MASKED_CASES, PACKED_SCALE_CASES, load_gemm_case
from oracle import cdg_oracle as oracle


def test_oracle_matches_reference_gemm(gemm_case):
    c = gemm_case
    d = torch.full_like(c["d"], 7.0)
    a = (c["a"], c["sa"]) if c["sa"] is not None else c["a"]
    oracle.m_grouped_fp8_fp4_gemm_nt_contiguous(a, (c["b"], c["sb"]), d, c["m_indices"])
    assert torch.equal(d.view(torch.int16) if d.dtype == torch.bfloat16 else d,
                       c["d"].view(torch.int16) if d.dtype == torch.bfloat16 else c["d"]), c["name"]


@pytest.mark.parametrize("name", MASKED_CASES)
def test_oracle_masked_matches_reference(name):
    c = load_gemm_case(name)
    assert c["masked"]
    d = torch.full_like(c["d"], 7.0)
    a = (c["a"], c["sa"]) if c["sa"] is not None else c["a"]
    oracle.m_grouped_fp8_fp4_gemm_nt_masked(a, (c["b"], c["sb"]), d, c["m_indices"])
    assert torch.equal(d.view(torch.int16), c["d"].view(torch.int16)), name


@pytest.mark.parametrize("name", PACKED_SCALE_CASES)
def test_packed_scale_fixtures(name):
    """Packed words unpack to the FP32 powers of two the reference consumed; the oracle reproduces D."""
    c = load_gemm_case(name)
    words = c["sa_packed"].to(torch.int64) & 0xFFFFFFFF
    kb = c["sa"].shape[1]
    e = torch.stack([(words >> (8 * i)) & 0xFF for i in range(4)], dim=2).reshape(words.shape[0], -1)[:, :kb]
    assert torch.equal(torch.pow(2.0, e.float() - 127.0), c["sa"])
    d = torch.full_like(c["d"], 7.0)
    oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((c["a"], c["sa"]), (c["b"], c["sb"]), d, c["m_indices"])
    assert torch.equal(d.view(torch.int16), c["d"].view(torch.int16)), name


def test_oracle_mega_moe_transform():
    z = _z("mega_moe_transform")
    (w1, s1), (w2, s2) = oracle.transform_weights_for_mega_moe((z["w1"], z["s1"]), (z["w2"], z["s2"]))
    for got, key in ((w1, "ow1"), (s1, "os1"), (w2, "ow2"), (s2, "os2")):
        assert np.array_equal(got, z[key]), key
    _, (w2b, s2b) = oracle.transform_weights_for_mega_moe((z["w1"], z["s1"]), (z["w2b"], z["s2b"]))
    assert np.array_equal(w2b, z["ow2b"]) and np.array_equal(s2b, z["os2b"])


def _z(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def test_oracle_sf_atom_reorder_bit_exact():
    for name in ("sf_reorder_arange", "sf_reorder_padded"):
        z = _z(name)
        assert np.array_equal(oracle.reorder_scale_to_sf_atom(z["src"]), z["dst"]), name


def test_oracle_fp4_dequant_all_bytes():
    z = _z("fp4_dequant_all_bytes")
    out = oracle.dequant_fp4_block(torch.from_numpy(z["src"]), torch.from_numpy(z["scale"]))
    assert np.array_equal(out.view(torch.int16).numpy(), z["dst"])


def test_oracle_float_scale_to_e8m0():
    z = _z("float_scale_to_e8m0")
    assert np.array_equal(oracle.float_scale_to_e8m0(torch.from_numpy(z["src"])).numpy(), z["dst"])


def test_known_answers_values():
    """The reference tests' literal expectations (tests/test_fp4_fallback.py:52,72; test_native_abi.py:290; test_scale_reorder.py:398)."""
    from conftest import load_gemm_case
    exp = {
        "kat_grouped_b": [5.0, 8.0, 0.0, 5.0],
        "kat_interleaved": [8.0, 5.0, 8.0, 5.0],
    }
    for name, col in exp.items():
        assert load_gemm_case(name)["d"][:, 0].float().tolist() == col
    assert bool((load_gemm_case("kat_all_128")["d"].float() == 128).all())
    assert bool((load_gemm_case("kat_scale_1536")["d"].float() == 1536).all())
    assert bool((load_gemm_case("kat_vllm_padding_zero")["d"].float() == 0).all())
