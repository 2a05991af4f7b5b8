"""The SageAttention2++ oracle against fixtures made by the reference itself (CPU only).

Given the reference's K mean (torch's fp32 mean), the oracle's INT8 Q/K
codes, per-row and per-key scales, FP8 V bytes and per-channel scales must be
bit-identical to the reference's, and its output must match the reference's
output to the last ulp of the output dtype on almost every element.
"""

from __future__ import annotations

import pytest
import torch
from conftest import load_sage_golden, sage_cases

from oracle import sage2pp


@pytest.mark.parametrize("name", sage_cases())
def test_oracle_codes_and_scales_match_reference(name: str) -> None:
    case = load_sage_golden(name)
    p = sage2pp.prepare(case["query"], case["key"], case["value"], key_mean=case["key_mean"].numpy())
    assert torch.equal(p["query_int8"], case["query_int8"])
    assert torch.equal(p["query_scale"], case["query_scale"])
    assert torch.equal(p["key_int8"], case["key_int8"])
    assert torch.equal(p["key_scale"], case["key_scale"])
    assert torch.equal(p["value_fp8"], case["value_fp8"])
    assert torch.equal(p["value_scale"], case["value_scale"])


@pytest.mark.parametrize("name", sage_cases())
def test_oracle_output_matches_reference(name: str) -> None:
    case = load_sage_golden(name)
    out, _ = sage2pp.sage_attention_2pp(case["query"], case["key"], case["value"], case["scale"],
                                        case["is_causal"], key_mean=case["key_mean"].numpy())
    mine = out.to(case["dtype"]).float()
    ref = case["out"].to(case["dtype"]).float()
    err = (mine - ref).abs()
    ulp = torch.finfo(case["dtype"]).eps * ref.abs().clamp_min(1e-3)
    assert (err <= 2 * ulp).all(), err.max().item()
    assert (err > 0).float().mean().item() < 1e-3


@pytest.mark.parametrize("name", sage_cases())
def test_exact_mean_codes_agree_with_reference(name: str) -> None:
    # With the oracle's own exact (fp64) K mean, codes sit on rounding
    # boundaries at most rarely: allow an off-by-one on a tiny fraction.
    case = load_sage_golden(name)
    p = sage2pp.prepare(case["query"], case["key"], case["value"])
    assert torch.equal(p["query_int8"], case["query_int8"])
    diff = (p["key_int8"].short() - case["key_int8"].short()).abs()
    assert diff.max().item() <= 1 and (diff > 0).float().mean().item() < 1e-3
