"""Execution-plan overrides and the offline tuner on the GPU (B200 only).

Every plan the tuner can try must compute the same attention: each candidate
(production or re-arm kernel, causal tile order, split-KV tail with 2..8 key
ranges over various tail sizes) is launched on the same prepared operands and
compared with the production plan (rounding-level differences only) and with
the oracle (the reference's GPU bounds).  Plans the kernels
cannot run are refused by the library before any launch.
"""

from __future__ import annotations

import pytest
import torch
from conftest import require_b200

from oracle import oracle
from piper_kernels import _native
from piper_kernels.attention.piper_attention.b200 import (
    default_execution_plan,
    launch_piper_attention,
    prepare_piper_attention,
)
from piper_kernels.tuning import MEASURED, candidate_plans, tune_piper_attention

pytestmark = pytest.mark.gpu


def _inputs(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=g).to(dtype)
    k = (torch.randn(shape, generator=g) + torch.randn(shape[:2] + (1, shape[3]), generator=g) * 2).to(dtype)
    v = (torch.randn(shape, generator=g) + torch.randn(shape[:2] + (1, shape[3]), generator=g)).to(dtype)
    return q, k, v


@pytest.mark.parametrize(("shape", "dtype", "causal"), [
    ((1, 5, 4096, 128), torch.bfloat16, False),
    ((2, 3, 1000, 128), torch.float16, False),
    ((1, 4, 2048, 128), torch.float16, True),
    ((1, 3, 1500, 64), torch.bfloat16, False),
])
def test_every_candidate_plan_computes_the_same_attention(shape, dtype, causal) -> None:
    dev = require_b200()
    q, k, v = _inputs(shape, dtype, sum(shape))
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    d = shape[3]
    with torch.no_grad():
        prepared = prepare_piper_attention(qd, kd, vd, causal)
        production = default_execution_plan(prepared)
        base = launch_piper_attention(prepared, d**-0.5)
        plans = candidate_plans(production, rearm=[False, True], heavy_first=[False, True],
                                split_k=None if causal else [0, 2, 3, 8])
        outs = []
        for plan in plans:
            outs.append((plan, launch_piper_attention(prepared, d**-0.5, plan=plan).clone()))
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    expected = oracle.piper_attention_torch(q, k, v, d**-0.5, causal).float()
    for plan, out in outs:
        err = (out.float() - base.float()).abs()
        assert err.max().item() < 0.02 and err.mean().item() < 2e-4, (plan, err.max().item())
        if (plan.split_k, plan.tail_tiles, plan.rearm) == (production.split_k, production.tail_tiles,
                                                            production.rearm):
            # The tile order changes no arithmetic.  (The re-arm kernel takes
            # its lazy-rescale decision per 64-key block, the production
            # kernel per 128-key iteration: the same codes, but a rescale may
            # land before or after a block's PV product, which moves fp32 and
            # fp16 roundings; the bounds above cover that.)
            assert torch.equal(out, base), plan
        ref_err = (out.float().cpu() - expected).abs()
        assert ref_err.mean().item() < 0.003 and ref_err.max().item() < 0.12, plan


def test_plans_the_kernels_cannot_run_are_refused() -> None:
    dev = require_b200()
    q, k, v = (t.to(dev) for t in _inputs((1, 2, 512, 64), torch.float16, 5))
    with torch.no_grad():
        prepared = prepare_piper_attention(q, k, v, True)
        production = default_execution_plan(prepared)
        with pytest.raises(ValueError, match="fixed by the kernels"):
            launch_piper_attention(prepared, 0.125, plan=production.__class__(**{**production.as_dict(), "stages": production.stages + 1}))
        with pytest.raises(ValueError, match="non-causal launches only"):
            launch_piper_attention(prepared, 0.125, plan=production.with_choices(split_k=2, tail_tiles=1))


def test_tuner_selects_a_measured_candidate() -> None:
    dev = require_b200()
    q, k, v = (t.to(dev) for t in _inputs((1, 5, 4096, 128), torch.bfloat16, 9))
    with torch.no_grad():
        prepared = prepare_piper_attention(q, k, v, False)
        production = default_execution_plan(prepared)
    run = tune_piper_attention(q, k, v, candidates=candidate_plans(production, split_k=[0, 2, 4]),
                               warmup_ms=5, measurement_time_ms=20)
    assert all(r.status == MEASURED for r in run.records)
    assert run.selected is not None and run.selected.quality.sqnr_db > 30
