"""Benchmark records for the B200 backend in the reference's record format.

The reference's benchmark tooling (Piper Kernels 0.2.1,
``benchmarks/lib/reporting.py:18-70``, ``timing.py``, ``quality.py``,
``environment.py``, ``benchmark_attention.py:374-383``) writes one
versioned record per provider and shape:

    {"schema_version": 1, "benchmark": "attention", "provider": ...,
     "shape": {...}, "configuration": {...}, "timings": {...},
     "quality": {...}, "environment": {...}, "extra": {...}}

This module produces the same fields for the sm_100a operators
(``piper_attention`` and ``sage_attention_2pp``), so records of both
implementations can be compared key by key.  The standard phases are:

* ``first_call_ms``: the synchronized first call of the operator;
* ``preparation``: the quantization prepass (synchronized wall clock);
* ``prepared_execution``: the fused attention kernel on prepared operands
  (CUDA events on the launching stream);
* ``operator_end_to_end``: the whole operator call (synchronized wall
  clock).

Each timing is a median with its 20th and 80th percentiles over repeated
runs filling ``measurement_time_ms``.  Quality compares the output with a
float32 reference (PyTorch SDPA by default) in float64 arithmetic.

Command line (one JSON Lines record per operator and sequence length):

    python -m piper_kernels.benchmarking --heads 24 --sequence 4096 16384 \\
        --operator piper_attention sage_attention_2pp --output records.jsonl
"""

from __future__ import annotations

import argparse
import json
import math
import os
import platform
import subprocess
import sys
import time
from collections.abc import Callable, Mapping
from dataclasses import dataclass, field
from datetime import UTC, datetime
from pathlib import Path
from typing import Any

import torch

SCHEMA_VERSION = 1
PROVIDER = "piper_b200"
SAGE_PROVIDER = "sage_attention_2pp_b200"
DEVICE_EVENT = "device_event"
SYNCHRONIZED_WALL = "synchronized_wall"


def linear_quantile(ordered: list[float], q: float) -> float:
    """Quantile of a sorted, non-empty sample with linear interpolation."""
    if not ordered:
        raise ValueError("empty sample")
    pos = (len(ordered) - 1) * q
    lo, hi = math.floor(pos), math.ceil(pos)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (pos - lo)


@dataclass(frozen=True)
class Timing:
    """Median latency with its 20th/80th percentiles, in milliseconds."""

    median_ms: float
    p20_ms: float
    p80_ms: float
    clock: str

    @classmethod
    def from_samples(cls, samples: list[float], clock: str) -> "Timing":
        s = sorted(samples)
        return cls(linear_quantile(s, 0.5), linear_quantile(s, 0.2), linear_quantile(s, 0.8), clock)

    def as_dict(self) -> dict[str, float | str]:
        return {"median_ms": self.median_ms, "p20_ms": self.p20_ms, "p80_ms": self.p80_ms, "clock": self.clock}


@dataclass(frozen=True)
class PhaseTimings:
    warmup_ms: int
    measurement_time_ms: int
    first_call_ms: float | None
    preparation: Timing | None
    prepared_execution: Timing
    operator_end_to_end: Timing | None

    def as_dict(self) -> dict[str, Any]:
        return {
            "warmup_ms": self.warmup_ms,
            "measurement_time_ms": self.measurement_time_ms,
            "first_call_ms": self.first_call_ms,
            "first_call_clock": None if self.first_call_ms is None else SYNCHRONIZED_WALL,
            "preparation": None if self.preparation is None else self.preparation.as_dict(),
            "prepared_execution": self.prepared_execution.as_dict(),
            "operator_end_to_end": None if self.operator_end_to_end is None else self.operator_end_to_end.as_dict(),
        }


@dataclass(frozen=True)
class Saturation:
    """How many quantized values sit at the two ends of their range."""

    minimum_count: int
    maximum_count: int
    total_count: int

    def as_dict(self) -> dict[str, int | float]:
        count = self.minimum_count + self.maximum_count
        return {
            "minimum_count": self.minimum_count,
            "maximum_count": self.maximum_count,
            "count": count,
            "total_count": self.total_count,
            "fraction": count / self.total_count if self.total_count else 0.0,
        }


def measure_saturation(values: torch.Tensor, minimum: int, maximum: int) -> Saturation:
    return Saturation(int((values == minimum).sum().item()), int((values == maximum).sum().item()), values.numel())


@dataclass(frozen=True)
class QualityMetrics:
    mean_absolute_error: float
    max_absolute_error: float
    relative_l1_error: float
    relative_l2_error: float
    sqnr_db: float
    cosine_similarity: float
    actual_nonfinite_count: int
    reference_nonfinite_count: int
    nonfinite_mismatch_count: int
    saturation: Mapping[str, Saturation] = field(default_factory=dict)

    def as_dict(self) -> dict[str, Any]:
        return {
            "mean_absolute_error": self.mean_absolute_error,
            "max_absolute_error": self.max_absolute_error,
            "relative_l1_error": self.relative_l1_error,
            "relative_l2_error": self.relative_l2_error,
            "sqnr_db": self.sqnr_db,
            "cosine_similarity": self.cosine_similarity,
            "actual_nonfinite_count": self.actual_nonfinite_count,
            "reference_nonfinite_count": self.reference_nonfinite_count,
            "nonfinite_mismatch_count": self.nonfinite_mismatch_count,
            "saturation": {k: v.as_dict() for k, v in self.saturation.items()},
        }


def measure_quality(actual: torch.Tensor, reference: torch.Tensor,
                    saturation: Mapping[str, Saturation] | None = None) -> QualityMetrics:
    """Error metrics over the pairs that are finite in both, in float64.

    (float32 reductions over millions of outputs near one drift by percents,
    so everything is accumulated in float64.)
    """
    if actual.shape != reference.shape:
        raise ValueError(f"shape mismatch: {tuple(actual.shape)} vs {tuple(reference.shape)}")
    a = actual.detach().to(torch.float64).flatten()
    r = reference.detach().to(torch.float64).flatten()
    fa, fr = torch.isfinite(a), torch.isfinite(r)
    both = fa & fr
    a, r = a[both], r[both]
    err = a - r
    n = max(a.numel(), 1)
    err_l1 = err.abs().sum()
    err_l2 = torch.linalg.vector_norm(err)
    ref_l1 = r.abs().sum().clamp_min(torch.finfo(torch.float64).tiny)
    ref_l2 = torch.linalg.vector_norm(r)
    act_l2 = torch.linalg.vector_norm(a)
    if act_l2 == 0 or ref_l2 == 0:
        cosine = 1.0 if act_l2 == 0 and ref_l2 == 0 else 0.0
    else:
        cosine = float((torch.dot(a, r) / (act_l2 * ref_l2)).clamp(-1, 1))
    sqnr = float(20 * torch.log10(ref_l2 / err_l2)) if err_l2 > 0 else float("inf")
    return QualityMetrics(
        mean_absolute_error=float(err_l1 / n),
        max_absolute_error=float(err.abs().max()) if err.numel() else 0.0,
        relative_l1_error=float(err_l1 / ref_l1),
        relative_l2_error=float(err_l2 / ref_l2.clamp_min(torch.finfo(torch.float64).tiny)),
        sqnr_db=sqnr,
        cosine_similarity=cosine,
        actual_nonfinite_count=int((~fa).sum()),
        reference_nonfinite_count=int((~fr).sum()),
        nonfinite_mismatch_count=int((fa != fr).sum()),
        saturation=dict(saturation or {}),
    )


def _git(args: list[str], cwd: Path) -> str | None:
    try:
        out = subprocess.run(["git", *args], cwd=cwd, capture_output=True, text=True, timeout=10)
    except (OSError, subprocess.TimeoutExpired):
        return None
    return out.stdout.strip() if out.returncode == 0 else None


def capture_environment(repo: Path | None = None, device: torch.device | None = None) -> dict[str, Any]:
    """Software, GPU and repository state (the reference's environment fields)."""
    repo = repo or Path(__file__).resolve().parents[2]
    try:
        import triton  # noqa: PLC0415

        triton_version = triton.__version__
    except ImportError:
        triton_version = None
    gpu_name = gpu_arch = driver = None
    index = None
    if torch.cuda.is_available():
        index = (device or torch.device("cuda", torch.cuda.current_device())).index
        props = torch.cuda.get_device_properties(index)
        gpu_name = props.name
        gpu_arch = f"sm_{props.major}{props.minor}"
        try:
            import pynvml  # noqa: PLC0415

            pynvml.nvmlInit()
            driver = pynvml.nvmlSystemGetDriverVersion()
            driver = driver.decode() if isinstance(driver, bytes) else driver
        except Exception:  # NVML absent: leave the driver unknown
            driver = None
    status = _git(["status", "--porcelain"], repo)
    return {
        "captured_at_utc": datetime.now(UTC).isoformat(),
        "python_version": sys.version.split()[0],
        "platform": platform.platform(),
        "torch_version": torch.__version__,
        "triton_version": triton_version,
        "accelerator_backend": "cuda" if torch.cuda.is_available() else None,
        "accelerator_runtime_version": torch.version.cuda,
        "accelerator_driver_version": driver,
        "gpu_name": gpu_name,
        "gpu_architecture": gpu_arch,
        "gpu_index": index,
        "git_revision": _git(["rev-parse", "HEAD"], repo),
        "git_dirty": None if status is None else bool(status),
    }


@dataclass(frozen=True)
class BenchmarkRecord:
    benchmark: str
    provider: str
    shape: Mapping[str, Any]
    configuration: Mapping[str, Any]
    timings: PhaseTimings
    environment: Mapping[str, Any]
    quality: QualityMetrics | None = None
    extra: Mapping[str, Any] = field(default_factory=dict)
    schema_version: int = SCHEMA_VERSION

    def as_dict(self) -> dict[str, Any]:
        return {
            "schema_version": self.schema_version,
            "benchmark": self.benchmark,
            "provider": self.provider,
            "shape": dict(self.shape),
            "configuration": dict(self.configuration),
            "timings": self.timings.as_dict(),
            "quality": None if self.quality is None else self.quality.as_dict(),
            "environment": dict(self.environment),
            "extra": dict(self.extra),
        }


def _json_safe(value: Any) -> Any:
    if isinstance(value, float) and not math.isfinite(value):
        return None
    if isinstance(value, Mapping):
        return {str(k): _json_safe(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_json_safe(v) for v in value]
    return value


def write_records(records: list[BenchmarkRecord], path: Path, fmt: str = "jsonl") -> None:
    """JSON Lines (one record per line) or one JSON array; non-finite floats become null."""
    rows = [_json_safe(r.as_dict()) for r in records]
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w") as f:
        if fmt == "jsonl":
            for row in rows:
                f.write(json.dumps(row, allow_nan=False) + "\n")
        else:
            json.dump(rows, f, allow_nan=False, indent=2)


def _wall_samples(fn: Callable[[], Any], warmup_ms: int, measurement_ms: int, sync: Callable[[], None]) -> list[float]:
    sync()
    t0 = time.perf_counter()
    while (time.perf_counter() - t0) * 1e3 < warmup_ms:
        fn()
        sync()
    samples: list[float] = []
    total = 0.0
    while total < measurement_ms:
        t = time.perf_counter()
        fn()
        sync()
        dt = (time.perf_counter() - t) * 1e3
        samples.append(dt)
        total += dt
    return samples


def _event_samples(fn: Callable[[], Any], warmup_ms: int, measurement_ms: int, stream) -> list[float]:
    _wall_samples(fn, warmup_ms, 1, torch.cuda.synchronize)
    samples: list[float] = []
    total = 0.0
    while total < measurement_ms:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        dt = e0.elapsed_time(e1)
        samples.append(dt)
        total += max(dt, 1e-3)
    return samples


def attention_shape(query: torch.Tensor, key: torch.Tensor) -> dict[str, int]:
    b, h, nq, d = query.shape
    return {"batch_size": b, "num_query_heads": h, "num_key_value_heads": h, "query_length": nq,
            "key_value_length": key.shape[2], "head_dim": d}


def effective_tflops(shape: Mapping[str, int], is_causal: bool, median_ms: float) -> float:
    """4*B*H*Nq*Nk*D / t (benchmark_attention.py's formula; causal counts visible pairs)."""
    b, h, nq, nk, d = (shape[k] for k in ("batch_size", "num_query_heads", "query_length", "key_value_length",
                                          "head_dim"))
    pairs = nq * (nq + 1) / 2 if is_causal else nq * nk
    return 4.0 * b * h * pairs * d / (median_ms * 1e-3) / 1e12


def sdpa_reference(query, key, value, scale: float, is_causal: bool) -> torch.Tensor:
    """Float32 scaled-dot-product attention, the reference's default quality target."""
    return torch.nn.functional.scaled_dot_product_attention(
        query.float(), key.float(), value.float(), is_causal=is_causal, scale=scale)


def _measure(query, key, value, *, operator: str, provider: str, is_causal: bool, scale: float | None,
             seed: int | None, warmup_ms: int, measurement_time_ms: int, reference: torch.Tensor | None,
             public: Callable, prepare: Callable, launch: Callable, saturation_of: Callable,
             configuration: Mapping[str, Any]) -> BenchmarkRecord:
    scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    stream = torch.cuda.current_stream(query.device)
    sync = torch.cuda.synchronize
    with torch.no_grad():
        sync()
        t = time.perf_counter()
        out = public(query, key, value, scale=scale, is_causal=is_causal)
        sync()
        first_ms = (time.perf_counter() - t) * 1e3
        prep = Timing.from_samples(_wall_samples(lambda: prepare(query, key, value, is_causal),
                                                 warmup_ms, measurement_time_ms, sync), SYNCHRONIZED_WALL)
        prepared = prepare(query, key, value, is_causal)
        buf = torch.empty_like(query, memory_format=torch.contiguous_format)
        run = Timing.from_samples(_event_samples(lambda: launch(prepared, scale, out=buf),
                                                 warmup_ms, measurement_time_ms, stream), DEVICE_EVENT)
        e2e = Timing.from_samples(_wall_samples(lambda: public(query, key, value, scale=scale, is_causal=is_causal),
                                                warmup_ms, measurement_time_ms, sync), SYNCHRONIZED_WALL)
        expected = sdpa_reference(query, key, value, scale, is_causal) if reference is None else reference
        quality = measure_quality(out, expected.to(out.device), saturation_of(prepared, key.shape[2]))
    shape = attention_shape(query, key)
    config = {
        "dtype": str(query.dtype).replace("torch.", ""),
        "is_causal": is_causal,
        "scale": scale,
        "seed": seed,
        "implementation": "sm100a_cuda",
        "algorithm": operator,
        **configuration,
    }
    return BenchmarkRecord(
        benchmark="attention",
        provider=provider,
        shape=shape,
        configuration=config,
        timings=PhaseTimings(warmup_ms, measurement_time_ms, first_ms, prep, run, e2e),
        environment=capture_environment(device=query.device),
        quality=quality,
        extra={"effective_tflops": effective_tflops(shape, is_causal, run.median_ms)},
    )


def measure_piper_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
                            is_causal: bool = False, scale: float | None = None, seed: int | None = None,
                            warmup_ms: int = 100, measurement_time_ms: int = 500,
                            reference: torch.Tensor | None = None) -> BenchmarkRecord:
    """One record for ``piper_attention`` on CUDA inputs (the phases of the module docstring)."""
    from . import piper_attention
    from .attention.piper_attention.b200 import launch_piper_attention, prepare_piper_attention

    def saturation_of(prepared, nk: int) -> dict[str, Saturation]:
        return {
            "query_int8": measure_saturation(prepared.query_int8, -127, 127),
            "key_int8": measure_saturation(prepared.key_int8, -127, 127),
            "value_int8": measure_saturation(prepared.value_int8_transposed[..., :nk], -127, 127),
        }

    return _measure(query, key, value, operator="piper_attention", provider=PROVIDER, is_causal=is_causal,
                    scale=scale, seed=seed, warmup_ms=warmup_ms, measurement_time_ms=measurement_time_ms,
                    reference=reference, public=piper_attention, prepare=prepare_piper_attention,
                    launch=launch_piper_attention, saturation_of=saturation_of,
                    configuration={"qk_quantization": "per_warp", "probability_dtype": "uint8",
                                   "value_dtype": "int8", "value_scale": "per_key"})


def measure_sage_attention_2pp(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
                               is_causal: bool = False, scale: float | None = None, seed: int | None = None,
                               warmup_ms: int = 100, measurement_time_ms: int = 500,
                               reference: torch.Tensor | None = None) -> BenchmarkRecord:
    """One record for ``sage_attention_2pp`` (configuration keys of the reference's Sage provider)."""
    from . import sage_attention_2pp
    from .attention.sage_attention_2pp.b200 import launch_sage_attention_2pp, prepare_sage_attention_2pp

    def saturation_of(prepared, _nk: int) -> dict[str, Saturation]:
        return {
            "query_int8": measure_saturation(prepared.query_int8, -127, 127),
            "key_int8": measure_saturation(prepared.key_int8, -127, 127),
        }

    return _measure(query, key, value, operator="sage_attention_2pp", provider=SAGE_PROVIDER,
                    is_causal=is_causal, scale=scale, seed=seed, warmup_ms=warmup_ms,
                    measurement_time_ms=measurement_time_ms, reference=reference, public=sage_attention_2pp,
                    prepare=prepare_sage_attention_2pp, launch=launch_sage_attention_2pp,
                    saturation_of=saturation_of,
                    configuration={"qk_quantization": "per_thread", "probability_dtype": "float8_e4m3fn",
                                   "value_dtype": "float8_e4m3fn", "value_scale": "per_channel",
                                   "pv_accumulation": "fp32", "block_n": 64})


MEASURES = {"piper_attention": measure_piper_attention, "sage_attention_2pp": measure_sage_attention_2pp}


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--operator", choices=sorted(MEASURES), nargs="+", default=["piper_attention"])
    parser.add_argument("--batch-size", type=int, default=1)
    parser.add_argument("--heads", type=int, default=24)
    parser.add_argument("--sequence", type=int, nargs="+", default=[4096])
    parser.add_argument("--kv-sequence", type=int, default=None)
    parser.add_argument("--head-dim", type=int, default=128)
    parser.add_argument("--dtype", choices=["float16", "bfloat16"], default="bfloat16")
    parser.add_argument("--causal", action="store_true")
    parser.add_argument("--scale", type=float, default=None)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--warmup-ms", type=int, default=100)
    parser.add_argument("--measurement-time-ms", type=int, default=500)
    parser.add_argument("--output", type=Path, default=None)
    parser.add_argument("--format", choices=["jsonl", "json"], default="jsonl")
    args = parser.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    dtype = getattr(torch, args.dtype)
    records = []
    for n in args.sequence:
        nk = args.kv_sequence or n
        g = torch.Generator(device=dev).manual_seed(args.seed)
        q = torch.randn((args.batch_size, args.heads, n, args.head_dim), generator=g, device=dev).to(dtype)
        k = torch.randn((args.batch_size, args.heads, nk, args.head_dim), generator=g, device=dev).to(dtype)
        v = torch.randn((args.batch_size, args.heads, nk, args.head_dim), generator=g, device=dev).to(dtype)
        for operator in args.operator:
            rec = MEASURES[operator](q, k, v, is_causal=args.causal, scale=args.scale, seed=args.seed,
                                     warmup_ms=args.warmup_ms, measurement_time_ms=args.measurement_time_ms)
            records.append(rec)
            t = rec.timings
            print(f"{rec.provider} N={n}: prepared {t.prepared_execution.median_ms:.3f} ms "
                  f"({rec.extra['effective_tflops']:.1f} TFLOPS-equivalent), end-to-end "
                  f"{t.operator_end_to_end.median_ms:.3f} ms, SQNR {rec.quality.sqnr_db:.1f} dB", flush=True)
    if args.output is not None:
        write_records(records, args.output, args.format)


if __name__ == "__main__":
    os.environ.setdefault("PYTHONUNBUFFERED", "1")
    main()
