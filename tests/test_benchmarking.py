"""Benchmark records in the reference's record format (CPU parts).

Field names follow the reference's versioned record
(benchmarks/lib/reporting.py:47-70, timing.py:56-95, quality.py:59-72,
environment.py:35-51), so records of both implementations compare key by key.
"""

from __future__ import annotations

import json
import math

import pytest
import torch

from piper_kernels import benchmarking as bm

TOP = {"schema_version", "benchmark", "provider", "shape", "configuration", "timings", "quality", "environment", "extra"}
TIMINGS = {"warmup_ms", "measurement_time_ms", "first_call_ms", "first_call_clock", "preparation",
           "prepared_execution", "operator_end_to_end"}
TIMING = {"median_ms", "p20_ms", "p80_ms", "clock"}
QUALITY = {"mean_absolute_error", "max_absolute_error", "relative_l1_error", "relative_l2_error", "sqnr_db",
           "cosine_similarity", "actual_nonfinite_count", "reference_nonfinite_count", "nonfinite_mismatch_count",
           "saturation"}
ENVIRONMENT = {"captured_at_utc", "python_version", "platform", "torch_version", "triton_version",
               "accelerator_backend", "accelerator_runtime_version", "accelerator_driver_version", "gpu_name",
               "gpu_architecture", "gpu_index", "git_revision", "git_dirty"}
SHAPE = {"batch_size", "num_query_heads", "num_key_value_heads", "query_length", "key_value_length", "head_dim"}


def test_quantiles_interpolate_linearly() -> None:
    assert bm.linear_quantile([1.0, 2.0, 3.0, 4.0, 5.0], 0.5) == 3.0
    assert bm.linear_quantile([1.0, 2.0, 3.0, 4.0, 5.0], 0.2) == pytest.approx(1.8)
    t = bm.Timing.from_samples([5.0, 1.0, 3.0, 2.0, 4.0], bm.DEVICE_EVENT)
    assert t.p20_ms <= t.median_ms <= t.p80_ms and t.median_ms == 3.0
    with pytest.raises(ValueError):
        bm.linear_quantile([], 0.5)


def test_quality_metrics() -> None:
    ref = torch.tensor([1.0, -2.0, 3.0, 4.0])
    same = bm.measure_quality(ref.clone(), ref)
    assert same.mean_absolute_error == 0 and same.cosine_similarity == 1.0 and math.isinf(same.sqnr_db)
    off = bm.measure_quality(ref + torch.tensor([0.0, 0.0, 0.5, -0.5]), ref)
    assert off.mean_absolute_error == pytest.approx(0.25)
    assert off.max_absolute_error == pytest.approx(0.5)
    assert off.relative_l1_error == pytest.approx(1.0 / 10.0)
    assert off.sqnr_db == pytest.approx(20 * math.log10(math.sqrt(30.0) / math.sqrt(0.5)))
    nan = bm.measure_quality(torch.tensor([1.0, float("nan"), 3.0]), torch.tensor([1.0, 2.0, float("inf")]))
    assert (nan.actual_nonfinite_count, nan.reference_nonfinite_count, nan.nonfinite_mismatch_count) == (1, 1, 2)
    codes = torch.tensor([-127, 0, 127, 127], dtype=torch.int8)
    sat = bm.measure_saturation(codes, -127, 127).as_dict()
    assert sat == {"minimum_count": 1, "maximum_count": 2, "count": 3, "total_count": 4, "fraction": 0.75}
    with pytest.raises(ValueError, match="shape mismatch"):
        bm.measure_quality(torch.zeros(2), torch.zeros(3))


def test_record_has_the_reference_schema(tmp_path) -> None:
    t = bm.Timing(1.0, 0.9, 1.1, bm.DEVICE_EVENT)
    rec = bm.BenchmarkRecord(
        benchmark="attention", provider=bm.PROVIDER,
        shape=bm.attention_shape(torch.empty(1, 2, 64, 128), torch.empty(1, 2, 80, 128)),
        configuration={"dtype": "bfloat16", "is_causal": False},
        timings=bm.PhaseTimings(100, 500, 12.0, t, t, None),
        environment=bm.capture_environment(),
        quality=bm.measure_quality(torch.ones(4), torch.ones(4)),
        extra={"effective_tflops": 1.0},
    )
    d = rec.as_dict()
    assert set(d) == TOP and d["schema_version"] == 1
    assert set(d["timings"]) == TIMINGS and set(d["timings"]["prepared_execution"]) == TIMING
    assert d["timings"]["operator_end_to_end"] is None and d["timings"]["first_call_clock"] == bm.SYNCHRONIZED_WALL
    assert set(d["quality"]) == QUALITY and set(d["environment"]) == ENVIRONMENT and set(d["shape"]) == SHAPE
    assert d["shape"]["key_value_length"] == 80
    out = tmp_path / "r.jsonl"
    bm.write_records([rec, rec], out)
    rows = [json.loads(line) for line in out.read_text().splitlines()]
    assert len(rows) == 2 and rows[0]["quality"]["sqnr_db"] is None  # inf -> null, strict JSON
    bm.write_records([rec], tmp_path / "r.json", "json")
    assert json.loads((tmp_path / "r.json").read_text())[0]["provider"] == bm.PROVIDER


def test_effective_tflops_formula() -> None:
    shape = {"batch_size": 1, "num_query_heads": 2, "query_length": 1000, "key_value_length": 1000, "head_dim": 128}
    assert bm.effective_tflops(shape, False, 1.0) == pytest.approx(4 * 2 * 1000 * 1000 * 128 / 1e-3 / 1e12)
    assert bm.effective_tflops(shape, True, 1.0) == pytest.approx(4 * 2 * 1000 * 1001 / 2 * 128 / 1e-3 / 1e12)


def test_both_operators_have_record_producers() -> None:
    assert set(bm.MEASURES) == {"piper_attention", "sage_attention_2pp"}
    assert bm.MEASURES["piper_attention"] is bm.measure_piper_attention
    assert bm.MEASURES["sage_attention_2pp"] is bm.measure_sage_attention_2pp
    assert bm.PROVIDER != bm.SAGE_PROVIDER


def test_cli_rejects_an_unknown_operator() -> None:
    with pytest.raises(SystemExit):
        bm.main(["--operator", "flash_attention"])
