"""Quantization prepass on the GPU vs the oracle and the reference (B200 only).

Codes and scales are integer/byte work: they must be bit-exact.  The sequence
means are computed on both sides with an exact fp64 sum rounded once to fp32,
so they match exactly too; the codes are compared both against the oracle run
on the GPU's own means and end to end.  The golden fixtures (made by the
reference itself) are checked as well.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_cases, load_golden, require_b200

from oracle import oracle
from piper_kernels import _native
from piper_kernels.attention.piper_attention.b200 import prepare_piper_attention

pytestmark = pytest.mark.gpu


def _check_against_oracle(q, k, v, is_causal) -> None:
    dev = require_b200()
    prepared = prepare_piper_attention(q.to(dev), k.to(dev), v.to(dev), is_causal)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    km = prepared.key_mean.cpu().numpy()
    vm = prepared.value_mean.cpu().numpy()
    ref = oracle.prepare(q, k, v, is_causal, key_mean=km, value_mean=None if is_causal else vm)
    own = oracle.prepare(q, k, v, is_causal)
    assert np.array_equal(km, own.key_mean)
    if is_causal:
        assert not vm.any()
    else:
        assert np.array_equal(vm, own.value_mean)
    assert np.array_equal(prepared.query_int8.cpu().numpy(), ref.query_int8)
    assert np.array_equal(prepared.query_scale.cpu().numpy(), ref.query_scale)
    assert np.array_equal(prepared.key_int8.cpu().numpy(), ref.key_int8)
    assert np.array_equal(prepared.key_scale.cpu().numpy(), ref.key_scale)
    assert np.array_equal(prepared.value_int8.cpu().numpy(), ref.value_int8)
    assert np.array_equal(prepared.value_scale.cpu().numpy(), ref.value_scale)
    vt = prepared.value_int8_transposed.cpu()
    nk = k.shape[2]
    assert not vt[..., nk:].any(), "padded keys must hold zero codes"
    # The stored operand is fp16 and must hold the INT8 codes exactly.
    vf = prepared.value_f16_transposed.cpu().float()
    assert torch.equal(vf, vt.float())


@pytest.mark.parametrize("name", golden_cases())
def test_prepass_matches_oracle_on_golden_inputs(name: str) -> None:
    case = load_golden(name)
    _check_against_oracle(case["query"], case["key"], case["value"], case["is_causal"])


@pytest.mark.parametrize("name", golden_cases())
def test_prepass_codes_match_reference_fixtures(name: str) -> None:
    dev = require_b200()
    case = load_golden(name)
    prepared = prepare_piper_attention(case["query"].to(dev), case["key"].to(dev), case["value"].to(dev),
                                       case["is_causal"])
    assert np.array_equal(prepared.query_int8.cpu().numpy(), case["query_int8"])
    assert np.array_equal(prepared.query_scale.cpu().numpy(), case["query_scale"])
    # K and V codes depend on the means, which torch sums in fp32: allow the
    # rare code that sits on a rounding boundary to differ by one.
    for mine, ref in ((prepared.key_int8, case["key_int8"]), (prepared.value_int8, case["value_int8"])):
        diff = (mine.cpu().to(torch.int16) - torch.from_numpy(ref).to(torch.int16)).abs()
        assert diff.max().item() <= 1
        assert (diff > 0).float().mean().item() < 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("is_causal", [False, True])
@pytest.mark.parametrize("n", [1, 63, 1000, 2048])
def test_prepass_matches_oracle_on_random_shapes(dtype, head_dim, is_causal, n) -> None:
    g = torch.Generator().manual_seed(n + head_dim)
    q = torch.randn((2, 3, n, head_dim), generator=g).to(dtype)
    k = (torch.randn((2, 3, n, head_dim), generator=g) + torch.randn((2, 3, 1, head_dim), generator=g) * 3).to(dtype)
    v = (torch.randn((2, 3, n, head_dim), generator=g) + 0.5).to(dtype)
    _check_against_oracle(q, k, v, is_causal)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("amax", [1.0, 3.75, 127.0])
@pytest.mark.parametrize("is_causal", [False, True])
def test_prepass_rounding_over_every_representable_input(dtype, amax, is_causal) -> None:
    # Every finite value of the input type in [-amax, amax] is quantized, each
    # 32x128 block holding amax once so the query scale is fixed: every
    # quotient's rounding (near-ties included) is checked against the
    # oracle's IEEE division, for Q, K and V codes alike.
    patterns = torch.arange(-(1 << 15), 1 << 15, dtype=torch.int32).to(torch.int16).view(dtype)
    values = patterns[torch.isfinite(patterns) & (patterns.float().abs() <= amax)]
    per_block = 32 * 128 - 1
    blocks = -(-values.numel() // per_block)
    flat = torch.zeros(blocks * per_block, dtype=dtype)
    flat[: values.numel()] = values
    flat = flat.reshape(blocks, per_block)
    head = torch.full((blocks, 1), amax, dtype=dtype)
    q = torch.cat([head, flat], dim=1).reshape(1, 1, blocks * 32, 128)
    k = q.flip(2).contiguous()
    v = q.roll(17, dims=3).contiguous()
    _check_against_oracle(q, k, v, is_causal)


def test_prepass_rectangular_and_strided_inputs() -> None:
    dev = require_b200()
    g = torch.Generator().manual_seed(5)
    storage = torch.randn((3, 2, 300, 128), generator=g).to(torch.bfloat16)
    q = storage.permute(1, 0, 2, 3)[:, :, :200]           # permuted B/H, sliced N
    kv = torch.randn((2, 3, 777, 128), generator=g).to(torch.bfloat16)
    k, v = kv, (kv * 0.5 + 1.0)
    _check_against_oracle(q, k, v, False)
    # A misaligned base (offset by one row of a 130-wide buffer) uses the
    # element-wise load path.
    wide = torch.randn((1, 1, 64, 130), generator=g).to(torch.float16)
    q2 = wide[..., 1:65]
    assert q2.stride(-1) == 1
    k2 = torch.randn((1, 1, 64, 64), generator=g).to(torch.float16)
    _check_against_oracle(q2, k2, k2, False)
    assert dev.type == "cuda"


@pytest.mark.parametrize("is_causal", [False, True])
def test_prepass_row_strided_inputs(is_causal: bool) -> None:
    # [B, N, H, D] storage viewed as [B, H, N, D]: consecutive rows of one
    # head are H*D elements apart.  1100 rows give three 512-row column-sum
    # chunks (the last one ragged) and a ragged last 64-row tile.
    require_b200()
    g = torch.Generator().manual_seed(6)
    storage = torch.randn((2, 1100, 3, 128), generator=g).to(torch.bfloat16)
    q = storage.permute(0, 2, 1, 3)
    k = (storage * 0.5 + 2.0).permute(0, 2, 1, 3)
    v = (storage.roll(5, dims=3) - 1.0).permute(0, 2, 1, 3)
    assert q.stride(2) == 3 * 128
    _check_against_oracle(q, k, v, is_causal)
