"""Offline tuner for the B200 Piper Attention execution plan.

The counterpart of the reference's schedule search (Piper Kernels 0.2.1,
``benchmarks/tune_piper_attention.py:53-221`` with the shared candidate loop
``benchmarks/lib/tuning.py:270-363``): build a bounded Cartesian product of
candidate plans around the production plan, reject candidates whose output
fails a quality gate (SQNR against float32 SDPA, 20 dB by default, as the
reference's ``meets_minimum_sqnr``), time the survivors' prepared execution
with CUDA events, and select the fastest.  Offline only: the production plan
stays the one ``piper_b200_select_plan`` returns; the tuner reports whether
another plan wins on a shape.

The run-time choices of a plan are the axes: the S re-arm instance, the
causal tile order and the split-KV tail (``split_k`` key ranges over
``tail_tiles`` trailing tiles).  Candidates the kernels cannot run are
recorded as skipped with the library's reason.

Command line (one JSON Lines record per candidate)::

    python -m piper_kernels.tuning --heads 40 --sequence 16384 --split-k 0 2 3 4 6 8 \\
        --rearm 0 1 --output tuning.jsonl
"""

from __future__ import annotations

import argparse
import json
import sys
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from itertools import product
from pathlib import Path
from typing import Any

import torch

from .attention.piper_attention._policy import PiperAttentionExecutionPlan
from .benchmarking import QualityMetrics, Timing, _event_samples, measure_quality, sdpa_reference

MEASURED = "measured"
QUALITY_REJECTED = "quality_rejected"
SKIPPED = "skipped"
DEFAULT_MINIMUM_SQNR_DB = 20.0
MAX_CANDIDATES = 64


def meets_minimum_sqnr(quality: QualityMetrics, minimum_sqnr_db: float) -> bool:
    """Quality gate: finite outputs wherever the reference is finite, and SQNR at or above the floor."""
    return quality.nonfinite_mismatch_count == 0 and quality.sqnr_db >= minimum_sqnr_db


def plan_name(plan: PiperAttentionExecutionPlan) -> str:
    split = f"split{plan.split_k}x{plan.tail_tiles}" if plan.split_k else "nosplit"
    return f"{'rearm' if plan.rearm else 'regbias'}-{'heavyfirst' if plan.heavy_first else 'inorder'}-{split}"


def _axis(values: Sequence[Any] | None, production: Any) -> tuple[Any, ...]:
    """An explicit search axis, or just the production value."""
    return tuple(dict.fromkeys(values)) if values else (production,)


def candidate_plans(
    production: PiperAttentionExecutionPlan,
    *,
    rearm: Sequence[bool] | None = None,
    heavy_first: Sequence[bool] | None = None,
    split_k: Sequence[int] | None = None,
    tail_tiles: Sequence[int] | None = None,
    max_candidates: int = MAX_CANDIDATES,
) -> tuple[PiperAttentionExecutionPlan, ...]:
    """The bounded product of the given axes around ``production`` (production first).

    ``tail_tiles`` applies to split candidates; by default a split candidate
    cuts the production tail, or the last partial wave when production has no
    split, capped so that the split CTAs fit the workspace's split region.
    Duplicates are dropped; more than ``max_candidates`` is an error.
    """
    axes = (
        _axis(rearm, production.rearm),
        _axis(heavy_first, production.heavy_first),
        _axis(split_k, production.split_k),
        _axis(tail_tiles, None),
    )
    count = 1
    for axis in axes:
        count *= len(axis)
    if count > max_candidates:
        raise ValueError(f"{count} tuning candidates exceed the limit of {max_candidates}")
    plans: dict[str, PiperAttentionExecutionPlan] = {plan_name(production): production}
    for r, hf, k, tail in product(*axes):
        if k == 0:
            plan = production.with_choices(rearm=bool(r), heavy_first=bool(hf), split_k=0)
        else:
            plan = production.with_choices(rearm=bool(r), heavy_first=bool(hf), split_k=int(k),
                                           tail_tiles=int(tail) if tail else None)
        plans.setdefault(plan_name(plan), plan)
    return tuple(plans.values())


@dataclass(frozen=True)
class TuningRecord:
    name: str
    configuration: dict[str, Any]
    status: str
    timing: Timing | None = None
    quality: QualityMetrics | None = None
    reason: str | None = None
    selected: bool = False

    def as_dict(self) -> dict[str, Any]:
        return {
            "name": self.name,
            "configuration": self.configuration,
            "status": self.status,
            "timing": None if self.timing is None else self.timing.as_dict(),
            "quality": None if self.quality is None else {
                k: v for k, v in self.quality.as_dict().items() if k != "saturation"},
            "reason": self.reason,
            "selected": self.selected,
        }


@dataclass(frozen=True)
class TuningRun:
    tuning: str
    shape: dict[str, Any]
    records: tuple[TuningRecord, ...] = field(default_factory=tuple)

    @property
    def selected(self) -> TuningRecord | None:
        return next((r for r in self.records if r.selected), None)


def tune_candidates(
    candidates: Sequence[PiperAttentionExecutionPlan],
    run: Callable[[PiperAttentionExecutionPlan], torch.Tensor],
    *,
    measure: Callable[[Callable[[], torch.Tensor]], Timing],
    measure_candidate_quality: Callable[[torch.Tensor], QualityMetrics] | None = None,
    quality_gate: Callable[[QualityMetrics], bool] | None = None,
    shape: dict[str, Any] | None = None,
) -> TuningRun:
    """Gate, time and rank ``candidates``; the fastest measured one is selected.

    ``run(plan)`` launches the prepared attention with ``plan`` and returns
    its output; a ``ValueError`` from it (the library refusing the plan)
    records the candidate as skipped.  Other exceptions propagate.
    """
    if not candidates:
        raise ValueError("at least one tuning candidate is required")
    if quality_gate is not None and measure_candidate_quality is None:
        raise ValueError("a quality gate requires a quality measurement function")
    records: list[TuningRecord] = []
    for plan in candidates:
        name, config = plan_name(plan), plan.as_dict()
        try:
            output = run(plan)
        except ValueError as error:
            records.append(TuningRecord(name, config, SKIPPED, reason=str(error)))
            continue
        quality = measure_candidate_quality(output) if measure_candidate_quality is not None else None
        if quality is not None and quality_gate is not None and not quality_gate(quality):
            records.append(TuningRecord(name, config, QUALITY_REJECTED, quality=quality,
                                        reason="quality gate rejected candidate"))
            continue
        timing = measure(lambda plan=plan: run(plan))
        records.append(TuningRecord(name, config, MEASURED, timing=timing, quality=quality))
    measured = [r for r in records if r.status == MEASURED]
    if measured:
        winner = min(measured, key=lambda r: r.timing.median_ms)
        records[records.index(winner)] = TuningRecord(**{**winner.__dict__, "selected": True})
    return TuningRun("piper_attention_execution_plan", dict(shape or {}), tuple(records))


def tune_piper_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    is_causal: bool = False,
    scale: float | None = None,
    candidates: Sequence[PiperAttentionExecutionPlan] | None = None,
    minimum_sqnr_db: float = DEFAULT_MINIMUM_SQNR_DB,
    warmup_ms: int = 50,
    measurement_time_ms: int = 200,
) -> TuningRun:
    """Tune the plan of one shape on the query's GPU (prepared execution timed)."""
    from .attention.piper_attention.b200 import default_execution_plan, launch_piper_attention, prepare_piper_attention
    from .benchmarking import attention_shape

    scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    with torch.no_grad():
        prepared = prepare_piper_attention(query, key, value, is_causal)
        production = default_execution_plan(prepared)
        if candidates is None:
            candidates = candidate_plans(production)
        expected = sdpa_reference(query, key, value, scale, is_causal)
        out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
        stream = torch.cuda.current_stream(query.device)

        def run(plan: PiperAttentionExecutionPlan) -> torch.Tensor:
            return launch_piper_attention(prepared, scale, out=out, plan=plan)

        def measure(fn: Callable[[], torch.Tensor]) -> Timing:
            return Timing.from_samples(_event_samples(fn, warmup_ms, measurement_time_ms, stream), "device_event")

        return tune_candidates(
            candidates, run, measure=measure,
            measure_candidate_quality=lambda output: measure_quality(output, expected),
            quality_gate=lambda quality: meets_minimum_sqnr(quality, minimum_sqnr_db),
            shape={**attention_shape(query, key), "is_causal": is_causal, "dtype": str(query.dtype)},
        )


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--batch-size", type=int, default=1)
    parser.add_argument("--heads", type=int, default=40)
    parser.add_argument("--sequence", type=int, default=16384)
    parser.add_argument("--kv-sequence", type=int, default=None)
    parser.add_argument("--head-dim", type=int, choices=(64, 128), default=128)
    parser.add_argument("--dtype", choices=("float16", "bfloat16"), default="bfloat16")
    parser.add_argument("--causal", action="store_true")
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--rearm", type=int, nargs="*", choices=(0, 1))
    parser.add_argument("--heavy-first", type=int, nargs="*", choices=(0, 1))
    parser.add_argument("--split-k", type=int, nargs="*")
    parser.add_argument("--tail-tiles", type=int, nargs="*")
    parser.add_argument("--max-candidates", type=int, default=MAX_CANDIDATES)
    parser.add_argument("--minimum-sqnr-db", type=float, default=DEFAULT_MINIMUM_SQNR_DB)
    parser.add_argument("--warmup-ms", type=int, default=50)
    parser.add_argument("--measurement-time-ms", type=int, default=200)
    parser.add_argument("--output", type=Path, default=None)
    args = parser.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("Piper Attention tuning requires a B200 GPU")
    from .attention.piper_attention.b200 import default_execution_plan, prepare_piper_attention

    dev = torch.device("cuda")
    dtype = getattr(torch, args.dtype)
    nk = args.kv_sequence or args.sequence
    g = torch.Generator(device=dev).manual_seed(args.seed)
    q = torch.randn((args.batch_size, args.heads, args.sequence, args.head_dim), generator=g, device=dev).to(dtype)
    k = torch.randn((args.batch_size, args.heads, nk, args.head_dim), generator=g, device=dev).to(dtype)
    v = torch.randn((args.batch_size, args.heads, nk, args.head_dim), generator=g, device=dev).to(dtype)
    with torch.no_grad():
        production = default_execution_plan(prepare_piper_attention(q, k, v, args.causal))
    flags = {"rearm": args.rearm, "heavy_first": args.heavy_first}
    candidates = candidate_plans(
        production, rearm=[bool(x) for x in flags["rearm"]] if flags["rearm"] else None,
        heavy_first=[bool(x) for x in flags["heavy_first"]] if flags["heavy_first"] else None,
        split_k=args.split_k, tail_tiles=args.tail_tiles, max_candidates=args.max_candidates)
    run = tune_piper_attention(q, k, v, is_causal=args.causal, candidates=candidates,
                               minimum_sqnr_db=args.minimum_sqnr_db, warmup_ms=args.warmup_ms,
                               measurement_time_ms=args.measurement_time_ms)
    rows = [{"schema_version": 1, "tuning": run.tuning, "shape": run.shape, **r.as_dict()} for r in run.records]
    text = "\n".join(json.dumps(row, allow_nan=False) for row in rows) + "\n"
    if args.output is None:
        sys.stdout.write(text)
    else:
        args.output.write_text(text)


if __name__ == "__main__":
    main()
