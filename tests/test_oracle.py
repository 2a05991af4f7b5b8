"""Pin the CPU oracle to the reference (golden fixtures) -- CPU only.

The fixtures in tests/golden were produced by tests/golden/make_golden.py,
which runs the Piper Kernels 0.2.1 portable reference itself.  The oracle must
reproduce its codes and scales bit for bit when given the same sequence means,
its means to within a few fp32 ulps of the data's magnitude, and its outputs to
within one output-dtype ulp on almost every element.  The property tests mirror
tests/attention/piper_attention/test_reference.py of the reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_cases, load_golden

from oracle import oracle

oracle.build()


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_codes_and_scales_match_reference_bit_for_bit(name: str) -> None:
    case = load_golden(name)
    vmean = None if case["is_causal"] else case["value_mean"]
    p = oracle.prepare(case["query"], case["key"], case["value"], case["is_causal"],
                       key_mean=case["key_mean"], value_mean=vmean)
    assert np.array_equal(p.query_int8, case["query_int8"])
    assert np.array_equal(p.query_scale, case["query_scale"])
    assert np.array_equal(p.key_int8, case["key_int8"])
    assert np.array_equal(p.key_scale, case["key_scale"])
    assert np.array_equal(p.value_int8, case["value_int8"])
    assert np.array_equal(p.value_scale, case["value_scale"])


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_means_match_reference(name: str) -> None:
    case = load_golden(name)
    k = case["key"].float().numpy()
    mine = oracle.sequence_mean(k)
    # torch sums in fp32 (cascade); the oracle sums exactly and rounds once.
    bound = 8 * np.finfo(np.float32).eps * np.abs(k).max(axis=2)
    assert (np.abs(mine - case["key_mean"]) <= bound).all()
    if not case["is_causal"]:
        v = case["value"].float().numpy()
        bound_v = 8 * np.finfo(np.float32).eps * np.abs(v).max(axis=2)
        assert (np.abs(oracle.sequence_mean(v) - case["value_mean"]) <= bound_v).all()


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_output_matches_reference(name: str) -> None:
    case = load_golden(name)
    vmean = None if case["is_causal"] else case["value_mean"]
    out, _ = oracle.piper_attention(case["query"], case["key"], case["value"], case["scale"],
                                    case["is_causal"], key_mean=case["key_mean"], value_mean=vmean)
    mine = torch.from_numpy(out).to(case["dtype"]).float()
    ref = case["out"].float()
    diff = (mine - ref).abs()
    ulp = torch.finfo(case["dtype"]).eps * ref.abs().clamp_min(1.0)
    # exp/log come from different libm implementations: allow one output ulp
    # on a handful of elements, nothing more.
    assert (diff <= ulp).all()
    assert (diff > 0).float().mean().item() < 1e-3


def test_oracle_raw_codes_match_reference_on_every_case() -> None:
    """Without the reference's means, codes still match (means agree to the ulp)."""
    total = mismatched = 0
    for name in golden_cases():
        case = load_golden(name)
        p = oracle.prepare(case["query"], case["key"], case["value"], case["is_causal"])
        for mine, ref in ((p.key_int8, case["key_int8"]), (p.value_int8, case["value_int8"])):
            total += ref.size
            mismatched += int((mine != ref).sum())
    assert mismatched / total < 1e-4


@pytest.mark.parametrize("is_causal", [False, True])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_oracle_is_close_to_exact_attention(head_dim: int, is_causal: bool) -> None:
    # reference tests/attention/piper_attention/test_reference.py:9-39
    torch.manual_seed(51)
    q = torch.randn(1, 2, 65, head_dim, dtype=torch.bfloat16)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    actual = oracle.piper_attention_torch(q, k, v, head_dim**-0.5, is_causal)
    expected = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=is_causal)
    err = (actual.float() - expected.float()).abs()
    assert actual.dtype is q.dtype
    assert err.mean().item() < 0.01
    assert err.max().item() < 0.2


def test_oracle_restores_constant_value_exactly() -> None:
    # reference test_reference.py:42-57
    torch.manual_seed(52)
    q = torch.randn(1, 2, 65, 64, dtype=torch.float16)
    k = torch.randn_like(q)
    v = torch.randn(1, 2, 1, 64, dtype=torch.float16).expand_as(q).contiguous()
    actual = oracle.piper_attention_torch(q, k, v, 64**-0.5, False)
    torch.testing.assert_close(actual, v, atol=0.0, rtol=0.0)


def test_causal_oracle_ignores_future_value_rows() -> None:
    # reference test_reference.py:60-76
    torch.manual_seed(53)
    q = torch.randn(1, 1, 65, 64, dtype=torch.float16)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    changed = v.clone()
    changed[:, :, 32:] = torch.randn_like(changed[:, :, 32:]) * 32
    a = oracle.piper_attention_torch(q, k, v, 64**-0.5, True)
    b = oracle.piper_attention_torch(q, k, changed, 64**-0.5, True)
    torch.testing.assert_close(a[:, :, :32], b[:, :, :32], atol=0.0, rtol=0.0)


def test_oracle_quantizer_error_is_at_most_half_a_step() -> None:
    # reference tests/attention/test_qk_quantization.py:11-33 (per_warp)
    torch.manual_seed(70)
    q = torch.randn(2, 3, 35, 64, dtype=torch.float16)
    k = torch.randn(2, 3, 67, 64, dtype=torch.float16)
    p = oracle.prepare(q, k, k, True)
    qs = np.repeat(p.query_scale, 32, axis=2)[:, :, :35]
    ks = np.repeat(p.key_scale, 64, axis=2)[:, :, :67]
    kc = k.float().numpy() - p.key_mean[:, :, None, :]
    assert (np.abs(p.query_int8 * qs[..., None] - q.float().numpy()) <= qs[..., None] / 2 + 1e-6).all()
    assert (np.abs(p.key_int8 * ks[..., None] - kc) <= ks[..., None] / 2 + 1e-6).all()
