"""Fused attention on the GPU vs the oracle, the reference fixtures and SDPA (B200 only).

Tolerances are the reference's own GPU parity bounds against its portable
implementation (tests/attention/piper_attention/test_triton.py:139-145):
mean |err| < 0.003 and max |err| < 0.12, plus a cosine-similarity floor.
The kernel evaluates exp/log in base 2 with hardware approximations, so a
UINT8 probability code can land one step away from the oracle's; that is the
only source of difference.  Exact properties (constant V, causal future
independence) are checked exactly, as the reference does.
"""

from __future__ import annotations

import pytest
import torch
from conftest import golden_cases, load_golden, require_b200

from oracle import oracle
from piper_kernels import _native, piper_attention
from piper_kernels.attention.piper_attention.b200 import launch_piper_attention, prepare_piper_attention

pytestmark = pytest.mark.gpu

MEAN_ABS_TOL = 0.003  # test_triton.py:144
MAX_ABS_TOL = 0.12  # test_triton.py:145
COSINE_FLOOR = 0.9999


def _compare(actual: torch.Tensor, expected: torch.Tensor) -> None:
    a = actual.float().cpu()
    e = expected.float().cpu()
    assert torch.isfinite(a).all()
    err = (a - e).abs()
    assert err.mean().item() < MEAN_ABS_TOL, err.mean().item()
    assert err.max().item() < MAX_ABS_TOL, err.max().item()
    # fp64: an fp32 reduction over millions of near-1 outputs is itself off by percents.
    cos = torch.nn.functional.cosine_similarity(a.double().flatten(), e.double().flatten(), dim=0).item()
    assert cos > COSINE_FLOOR, cos


def _run(q, k, v, scale=None, is_causal=False):
    dev = require_b200()
    with torch.no_grad():
        out = piper_attention(q.to(dev), k.to(dev), v.to(dev), scale=scale, is_causal=is_causal)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    return out


@pytest.mark.parametrize("name", golden_cases())
def test_attention_matches_reference_fixtures(name: str) -> None:
    case = load_golden(name)
    scale = case["scale"] if bool(case["scale_given"]) else None
    out = _run(case["query"], case["key"], case["value"], scale, case["is_causal"])
    assert out.shape == case["query"].shape and out.dtype is case["dtype"]
    _compare(out, case["out"])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("is_causal", [False, True])
def test_attention_matches_oracle(dtype: torch.dtype, head_dim: int, is_causal: bool) -> None:
    # test_triton.py:111-145 (B1 H2 N193, seed 54)
    g = torch.Generator().manual_seed(54)
    q = torch.randn((1, 2, 193, head_dim), generator=g).to(dtype)
    k = torch.randn((1, 2, 193, head_dim), generator=g).to(dtype)
    v = torch.randn((1, 2, 193, head_dim), generator=g).to(dtype)
    out = _run(q, k, v, is_causal=is_causal)
    assert out.dtype is dtype
    _compare(out, oracle.piper_attention_torch(q, k, v, head_dim**-0.5, is_causal))


@pytest.mark.parametrize(("nq", "nk", "is_causal"), [(1, 1, False), (1, 1, True), (9, 11, False), (300, 77, False),
                                                    (1000, 1000, True), (2049, 2049, False), (129, 4100, False)])
def test_attention_ragged_lengths(nq: int, nk: int, is_causal: bool) -> None:
    g = torch.Generator().manual_seed(nq * 7 + nk)
    q = torch.randn((2, 2, nq, 128), generator=g).to(torch.bfloat16)
    k = (torch.randn((2, 2, nk, 128), generator=g) + torch.randn((2, 2, 1, 128), generator=g) * 2).to(torch.bfloat16)
    v = (torch.randn((2, 2, nk, 128), generator=g) + torch.randn((2, 2, 1, 128), generator=g)).to(torch.bfloat16)
    out = _run(q, k, v, is_causal=is_causal)
    _compare(out, oracle.piper_attention_torch(q, k, v, 128**-0.5, is_causal))


def test_centered_value_restores_constant_value_exactly() -> None:
    # test_triton.py:212-222
    g = torch.Generator().manual_seed(56)
    q = torch.randn((1, 2, 1024, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 2, 1024, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((1, 2, 1, 128), generator=g).to(torch.bfloat16).expand_as(q).contiguous()
    out = _run(q, k, v)
    torch.testing.assert_close(out.cpu(), v, atol=0.0, rtol=0.0)


def test_causal_output_is_independent_of_future_value_rows() -> None:
    # test_triton.py:225-242
    g = torch.Generator().manual_seed(62)
    q = torch.randn((1, 1, 65, 64), generator=g).to(torch.float16)
    k = torch.randn((1, 1, 65, 64), generator=g).to(torch.float16)
    v = torch.randn((1, 1, 65, 64), generator=g).to(torch.float16)
    changed = v.clone()
    changed[:, :, 32:] = torch.randn((1, 1, 33, 64), generator=g).to(torch.float16) * 32
    a = _run(q, k, v, is_causal=True)
    b = _run(q, k, changed, is_causal=True)
    torch.testing.assert_close(a[:, :, :32], b[:, :, :32], atol=0.0, rtol=0.0)


def test_large_value_scale_stays_finite() -> None:
    # test_triton.py:245-266
    dev = require_b200()
    q = torch.ones((1, 1, 64, 64), dtype=torch.float16)
    k = torch.ones_like(q)
    k[:, :, 0] = -1
    v = torch.ones_like(q)
    v[:, :, 0] = 40000
    prepared = prepare_piper_attention(q.to(dev), k.to(dev), v.to(dev), False)
    out = launch_piper_attention(prepared, 64**-0.5)
    assert torch.isfinite(prepared.value_scale).all()
    assert torch.isfinite(out).all()
    _compare(out, oracle.piper_attention_torch(q, k, v, 64**-0.5, False))


def test_biased_value_quality_vs_sdpa() -> None:
    # test_triton.py:269-282
    g = torch.Generator().manual_seed(57)
    q = torch.randn((1, 1, 1024, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 1, 1024, 128), generator=g).to(torch.bfloat16)
    offset = torch.linspace(-8, 8, 128).reshape(1, 1, 1, 128)
    v = (offset + torch.randn((1, 1, 1024, 128), generator=g) * 0.25).to(torch.bfloat16)
    out = _run(q, k, v)
    expected = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert (out.float().cpu() - expected).square().mean() < 1e-3


def test_strided_inputs_and_torch_compile() -> None:
    # test_triton.py:356-376: permuted inputs, fullgraph compile == eager.
    dev = require_b200()
    g = torch.Generator().manual_seed(60)
    qs = torch.randn((3, 2, 128, 64), generator=g).to(torch.float16).to(dev)
    ks = torch.randn((3, 2, 128, 64), generator=g).to(torch.float16).to(dev)
    vs = torch.randn((3, 2, 128, 64), generator=g).to(torch.float16).to(dev)
    q, k, v = (t.permute(1, 0, 2, 3) for t in (qs, ks, vs))

    def consumer(q, k, v):
        return -piper_attention(q, k, v)

    with torch.no_grad():
        eager = consumer(q, k, v)
        compiled = torch.compile(consumer, fullgraph=True)(q, k, v)
    assert torch.equal(eager, compiled)
    _compare(-eager, oracle.piper_attention_torch(q.cpu(), k.cpu(), v.cpu(), 64**-0.5, False))


def test_prepared_split_equals_one_shot_call() -> None:
    dev = require_b200()
    g = torch.Generator().manual_seed(61)
    q = torch.randn((1, 2, 700, 128), generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn((1, 2, 700, 128), generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn((1, 2, 700, 128), generator=g).to(torch.bfloat16).to(dev)
    with torch.no_grad():
        one = piper_attention(q, k, v, is_causal=True)
        prepared = prepare_piper_attention(q, k, v, True)
        two = launch_piper_attention(prepared, 128**-0.5)
        again = launch_piper_attention(prepared, 128**-0.5)
    assert torch.equal(one, two) and torch.equal(two, again)


@pytest.mark.parametrize(("shape", "dtype"), [((1, 2, 4096, 128), torch.bfloat16), ((1, 5, 16384, 128), torch.bfloat16),
                                              ((1, 1, 1000, 64), torch.float16)])
def test_split_tail_matches_unsplit_launch(shape, dtype) -> None:
    # The last partial wave's tiles are cut into key ranges whose partial
    # states a merge kernel combines; a workspace without the optional split
    # region runs the same problem unsplit.
    dev = require_b200()
    g = torch.Generator().manual_seed(sum(shape))
    q = torch.randn(shape, generator=g).to(dtype).to(dev)
    k = torch.randn(shape, generator=g).to(dtype).to(dev)
    v = (torch.randn(shape, generator=g) + 1).to(dtype).to(dev)
    b, h, n, d = shape
    layout = _native.workspace_layout(b, h, n, n, d)
    small = torch.empty(int(layout.split_state), dtype=torch.uint8, device=dev)
    with torch.no_grad():
        split = launch_piper_attention(prepare_piper_attention(q, k, v, False), d**-0.5)
        unsplit = launch_piper_attention(prepare_piper_attention(q, k, v, False, workspace=small), d**-0.5)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    err = (split.float() - unsplit.float()).abs()
    assert err.max().item() < 0.02 and err.mean().item() < 2e-4
    _compare(split, oracle.piper_attention_torch(q.cpu(), k.cpu(), v.cpu(), d**-0.5, False))


def test_benchmark_record_through_the_gpu() -> None:
    from piper_kernels import benchmarking as bm

    dev = require_b200()
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn((1, 4, 1024, 128), generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    rec = bm.measure_piper_attention(q, k, v, warmup_ms=5, measurement_time_ms=20).as_dict()
    t = rec["timings"]
    assert t["prepared_execution"]["clock"] == bm.DEVICE_EVENT and t["preparation"]["clock"] == bm.SYNCHRONIZED_WALL
    assert 0 < t["prepared_execution"]["p20_ms"] <= t["prepared_execution"]["median_ms"] <= t["prepared_execution"]["p80_ms"]
    assert rec["quality"]["sqnr_db"] > 25 and rec["quality"]["cosine_similarity"] > 0.999
    assert rec["environment"]["gpu_architecture"] == "sm_100" and rec["extra"]["effective_tflops"] > 0
