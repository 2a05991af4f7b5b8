"""Offline plan tuner: candidate enumeration, quality gate and selection -- CPU only.

The candidate loop takes its launch and timer as functions, so these tests
drive it with fakes (the reference's tuner tests do the same with fake
providers, ``tests/benchmarks/test_tuning.py``); the GPU run of the tuner is
in ``tests/test_gpu_tuning.py``.
"""

from __future__ import annotations

import pytest
import torch

from piper_kernels._targets import AcceleratorTarget
from piper_kernels.attention.piper_attention._policy import SPLIT_UNITS_MAX, select_execution_plan
from piper_kernels.benchmarking import Timing, measure_quality
from piper_kernels.tuning import (
    MEASURED,
    QUALITY_REJECTED,
    SKIPPED,
    candidate_plans,
    meets_minimum_sqnr,
    plan_name,
    tune_candidates,
)

B200 = AcceleratorTarget("cuda", "sm100", 148)


def _production(heads=40, n=16384, d=128, causal=False):
    return select_execution_plan(B200, batch=1, heads=heads, query_length=n, key_length=n, head_dim=d,
                                 is_causal=causal)


def test_production_only_by_default() -> None:
    prod = _production()
    assert candidate_plans(prod) == (prod,)


def test_product_of_axes_with_production_first() -> None:
    prod = _production()
    plans = candidate_plans(prod, rearm=[False, True], split_k=[0, 2, 3, 4])
    assert plans[0] == prod
    names = [plan_name(p) for p in plans]
    assert len(names) == len(set(names)) == 8
    for p in plans:
        if p.split_k:
            assert p.tail_tiles == 44 and p.ctas == 2560 - 44 + 44 * p.split_k
        else:
            assert p.tail_tiles == 0 and p.ctas == 2560


def test_split_candidates_on_an_unsplit_production_cut_the_last_partial_wave() -> None:
    prod = _production(heads=37, n=1024)  # 148 tiles: whole waves, no split
    assert prod.split_k == 0
    (split,) = [p for p in candidate_plans(prod, split_k=[0, 4]) if p.split_k]
    assert split.tail_tiles == min(148, SPLIT_UNITS_MAX // 4) and split.kernels == 2  # capped by the split region


def test_too_many_candidates_is_an_error() -> None:
    with pytest.raises(ValueError, match="exceed the limit"):
        candidate_plans(_production(), split_k=[0, 2, 3, 4, 5, 6, 7, 8], rearm=[False, True], max_candidates=8)


def test_gate_rejects_and_fastest_measured_wins() -> None:
    prod = _production()
    plans = candidate_plans(prod, split_k=[0, 2, 3, 4])
    reference = torch.linspace(-1, 1, 1000, dtype=torch.float64)
    noisy = reference + 0.5 * torch.sin(torch.arange(1000, dtype=torch.float64))  # SQNR far below 20 dB
    speed = {0: 3.0, 2: 2.0, 3: 1.0, 4: 0.5}

    def run(plan):
        if plan.split_k == 4:
            return noisy
        return reference + 1e-6

    def measure(fn):
        fn()
        return Timing(median_ms=current[0], p20_ms=current[0], p80_ms=current[0], clock="fake")

    current = [0.0]

    def run_and_note(plan):
        current[0] = speed[plan.split_k]
        return run(plan)

    result = tune_candidates(plans, run_and_note, measure=measure,
                             measure_candidate_quality=lambda out: measure_quality(out, reference),
                             quality_gate=lambda q: meets_minimum_sqnr(q, 20.0))
    status = {r.configuration["split_k"]: r.status for r in result.records}
    assert status == {0: MEASURED, 2: MEASURED, 3: MEASURED, 4: QUALITY_REJECTED}
    assert result.selected is not None and result.selected.configuration["split_k"] == 3
    assert sum(r.selected for r in result.records) == 1


def test_plans_the_library_refuses_are_skipped() -> None:
    prod = _production()

    def run(plan):
        if plan.split_k:
            raise ValueError("plan splits keys but the workspace has no split region")
        return torch.zeros(4)

    result = tune_candidates(candidate_plans(prod, split_k=[0, 3]), run,
                             measure=lambda fn: Timing(1.0, 1.0, 1.0, "fake"))
    statuses = sorted(r.status for r in result.records)
    assert statuses == [MEASURED, SKIPPED]
    assert result.selected.configuration["split_k"] == 0


def test_empty_candidates_and_gate_without_quality_are_errors() -> None:
    with pytest.raises(ValueError, match="at least one"):
        tune_candidates((), lambda p: None, measure=lambda fn: None)
    with pytest.raises(ValueError, match="quality measurement"):
        tune_candidates((_production(),), lambda p: None, measure=lambda fn: None, quality_gate=lambda q: True)
