"""Execution-plan policy on fake targets -- CPU only.

The plan is pure host logic in the C library (``piper_b200_select_plan``),
so, like the reference's policy tests
(``tests/attention/piper_attention/test_policy.py:18-21``), these build
targets by hand -- here sm_100 parts with different SM counts -- and check
the choices without a GPU.
"""

from __future__ import annotations

import pytest

from piper_kernels._targets import AcceleratorTarget
from piper_kernels.attention.piper_attention._policy import (
    SPLIT_UNITS_MAX,
    PiperAttentionExecutionPlan,
    select_execution_plan,
)

B200 = AcceleratorTarget("cuda", "sm100", 148)
SMALL = AcceleratorTarget("cuda", "sm100", 132)
UNSAID = AcceleratorTarget("cuda", "sm100")


def _select(target=B200, *, batch=1, heads=40, n=16384, nk=None, d=128, causal=False, split_region=True):
    return select_execution_plan(target, batch=batch, heads=heads, query_length=n, key_length=nk or n,
                                 head_dim=d, is_causal=causal, split_region=split_region)


def test_fixed_fields_report_the_compiled_kernels() -> None:
    for d, stages in ((128, 3), (64, 6)):
        plan = _select(d=d)
        assert (plan.tile_rows, plan.key_block, plan.stages) == (256, 64, stages)


def test_c4_plan_on_a_b200() -> None:
    plan = _select()
    # 40 heads x 64 tiles = 2560 tiles = 17 waves + 44 tiles on 148 SMs.
    assert plan.tiles == 2560 and plan.sms == 148
    assert plan.tail_tiles == 44 and plan.split_k == 3  # one wave of 132 third-tiles
    assert plan.ctas == 2560 - 44 + 44 * 3 and plan.kernels == 2
    assert not plan.rearm and not plan.heavy_first


def test_five_heads_per_gpu_fill_the_last_wave() -> None:
    # c4 split over 8 GPUs: 320 tiles = 2 waves + 24 tiles, each cut into 6 key ranges.
    plan = _select(heads=5)
    assert plan.tail_tiles == 24 and plan.split_k == 6 and plan.ctas == 296 + 144


def test_twenty_heads_per_gpu_split_into_two_waves_of_thirds() -> None:
    # c4 split over 2 GPUs: 1280 tiles = 8 waves + 96 tiles.  No k <= 148 / 96
    # helps, but k = 3 gives 288 third-tiles in two waves: 0.67 of a tile
    # instead of a whole wave.
    plan = _select(heads=20)
    assert plan.tail_tiles == 96 and plan.split_k == 3 and plan.ctas == 1184 + 288


def test_split_minimises_the_tail_in_tile_units() -> None:
    from math import ceil
    for heads in range(1, 80):
        plan = _select(heads=heads)
        tail = plan.tiles % 148
        cost = (lambda k: ceil(tail * k / 148) / k)
        best = min([1.0] + [cost(k) for k in range(2, 9) if tail * k <= SPLIT_UNITS_MAX])
        if plan.split_k == 0:
            assert tail == 0 or best == 1.0
        else:
            assert plan.tail_tiles == tail and abs(cost(plan.split_k) - best) < 1e-12
            assert all(cost(k) > best for k in range(2, plan.split_k))  # the smallest best k


def test_split_depends_on_the_sm_count() -> None:
    assert _select(SMALL).tail_tiles == 2560 % 132
    assert _select(UNSAID) == _select(B200)
    # Whole waves: no tail to split.
    assert _select(B200, heads=37, n=1024).split_k == 0  # 37 x 4 = 148 tiles


def test_causal_plan_has_no_split_and_heavy_tiles_first() -> None:
    plan = _select(batch=4, heads=32, n=8192, causal=True)
    assert plan.split_k == 0 and plan.tail_tiles == 0 and plan.kernels == 1
    assert plan.heavy_first


def test_tmem_probability_instance_everywhere() -> None:
    # The no-re-arm instance (probabilities in TMEM) is the production choice
    # for every head dimension and mask.
    assert not _select(d=128).rearm
    assert not _select(d=64).rearm
    assert not _select(d=128, causal=True).rearm


def test_no_split_without_the_workspace_region_or_short_keys() -> None:
    assert _select(split_region=False).split_k == 0
    # Two key blocks cannot be cut into more than one range of two blocks each.
    assert _select(heads=1, n=256, nk=128).split_k == 0


def test_with_choices_recomputes_derived_fields() -> None:
    plan = _select()
    unsplit = plan.with_choices(split_k=0)
    assert unsplit.tail_tiles == 0 and unsplit.ctas == plan.tiles and unsplit.kernels == 1
    wider = plan.with_choices(split_k=2)
    assert wider.tail_tiles == 44 and wider.ctas == 2560 - 44 + 88
    resplit = unsplit.with_choices(split_k=4)
    assert resplit.tail_tiles == 2560 % 148 and resplit.kernels == 2


def test_plan_round_trips_through_the_native_struct() -> None:
    plan = _select()
    assert PiperAttentionExecutionPlan.from_native(plan.to_native()) == plan


def test_invalid_plans_are_rejected() -> None:
    plan = _select()
    with pytest.raises(ValueError, match="split_k"):
        plan.with_choices(split_k=1)
    with pytest.raises(ValueError, match="tail_tiles"):
        PiperAttentionExecutionPlan(256, 64, 5, True, False, 0, 10, 3, 10, 1, 148)


def test_non_b200_targets_have_no_plan() -> None:
    with pytest.raises(ValueError, match="no B200 execution plan"):
        _select(AcceleratorTarget("cuda", "sm90", 132))
    with pytest.raises(ValueError, match="head_dim"):
        _select(d=96)
