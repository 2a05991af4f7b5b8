"""Host-side execution plan of the B200 Piper Attention kernels.

The counterpart of the reference's frozen launch policy (Piper Kernels 0.2.1,
``src/piper_kernels/attention/piper_attention/_policy.py:14-96``): a frozen
record of the launch choices for one call, selected per shape and target by
one function.  The selection itself lives in the C library
(``piper_b200_select_plan``) so that the native entry points and this module
cannot disagree; it is pure host logic, so tests drive it with fake targets
(other SM counts) on machines without a GPU, as the reference's policy tests
do (``tests/attention/piper_attention/test_policy.py:18-21``).

Fields (see ``piper_b200_plan_t``):

* ``tile_rows``, ``key_block``, ``stages`` -- fixed by the compiled kernels
  (two 128-row query tiles per CTA, 64-key softmax blocks, the depth of the
  production kernel's K/V shared-memory ring in 128-key iterations);
  reported, not chosen;
* ``rearm`` -- kernel: ``False`` is the production kernel (128 keys, two
  softmax blocks, per iteration with N = 128 QK^T MMAs; the INT32 scores
  converted with I2F; the probabilities written into TMEM over the spent scores, where
  the PV MMA reads them); ``True`` is the 64-key-block kernel that re-arms
  the INT32 score accumulators with the float bias pattern after each read
  and passes the probabilities to the PV MMA through shared memory;
* ``heavy_first`` -- causal launches schedule the query tiles with the most
  visible keys first;
* ``split_k`` / ``tail_tiles`` -- the split-KV tail: the trailing tiles of a
  partial last wave are cut into ``split_k`` key ranges whose partial states
  a merge kernel combines;
* ``tiles``, ``ctas``, ``kernels``, ``sms`` -- derived launch facts.
"""

from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass, replace

from ... import _native
from ..._targets import AcceleratorTarget

B200_SMS = 148
# Split-KV CTAs the workspace's split region holds at most (kMaxSplitUnits in
# the library's layout): tail_tiles * split_k may not exceed it.
SPLIT_UNITS_MAX = 512


@dataclass(frozen=True, slots=True)
class PiperAttentionExecutionPlan:
    """Launch choices for one Piper Attention call on sm_100a."""

    tile_rows: int
    key_block: int
    stages: int
    rearm: bool
    heavy_first: bool
    split_k: int
    tiles: int
    tail_tiles: int
    ctas: int
    kernels: int
    sms: int

    def __post_init__(self) -> None:
        if self.split_k < 0 or self.split_k == 1:
            raise ValueError("Piper Attention split_k must be 0 or at least 2")
        if (self.split_k == 0) != (self.tail_tiles == 0):
            raise ValueError("Piper Attention split_k and tail_tiles must both be zero or both positive")

    def as_dict(self) -> dict[str, object]:
        """Execution choices as serializable benchmark metadata."""
        return asdict(self)

    def with_choices(self, *, rearm: bool | None = None, heavy_first: bool | None = None,
                     split_k: int | None = None, tail_tiles: int | None = None) -> "PiperAttentionExecutionPlan":
        """A copy with some run-time choices changed (derived fields are recomputed at launch)."""
        changes: dict[str, object] = {}
        if rearm is not None:
            changes["rearm"] = rearm
        if heavy_first is not None:
            changes["heavy_first"] = heavy_first
        if split_k is not None:
            changes["split_k"] = split_k
            if split_k == 0:
                changes["tail_tiles"] = 0
            elif tail_tiles is None:
                tail = self.tail_tiles or self.tiles % self.sms or min(self.sms, self.tiles)
                changes["tail_tiles"] = max(1, min(tail, SPLIT_UNITS_MAX // split_k))
        if tail_tiles is not None:
            changes["tail_tiles"] = tail_tiles
        if "split_k" in changes or "tail_tiles" in changes:
            split = int(changes.get("split_k", self.split_k))
            tail = int(changes.get("tail_tiles", self.tail_tiles))
            changes["ctas"] = self.tiles - tail + tail * split
            changes["kernels"] = 2 if split else 1
        return replace(self, **changes)

    def to_native(self) -> _native.Plan:
        plan = _native.Plan()
        for name, value in self.as_dict().items():
            setattr(plan, name, int(value))
        return plan

    @classmethod
    def from_native(cls, plan: _native.Plan) -> "PiperAttentionExecutionPlan":
        return cls(
            tile_rows=plan.tile_rows, key_block=plan.key_block, stages=plan.stages, rearm=bool(plan.rearm),
            heavy_first=bool(plan.heavy_first), split_k=plan.split_k, tiles=plan.tiles, tail_tiles=plan.tail_tiles,
            ctas=plan.ctas, kernels=plan.kernels, sms=plan.sms,
        )


def select_execution_plan(
    target: AcceleratorTarget,
    *,
    batch: int,
    heads: int,
    query_length: int,
    key_length: int,
    head_dim: int,
    is_causal: bool,
    split_region: bool = True,
) -> PiperAttentionExecutionPlan:
    """The production plan for a problem on ``target``.

    ``target.multi_processor_count`` sizes the waves (148, a B200, when the
    target does not say).  ``split_region`` is whether the workspace holds
    the optional split-KV region (a full ``workspace_bytes`` workspace does).
    """
    if not target.supports_tcgen05_int8:
        raise ValueError(f"no B200 execution plan for target {target.backend}:{target.architecture}")
    sms = target.multi_processor_count or B200_SMS
    plan = _native.Plan()
    _native.check(
        _native.library().piper_b200_select_plan(batch, heads, query_length, key_length, head_dim,
                                                 1 if is_causal else 0, sms, 1 if split_region else 0,
                                                 ctypes.byref(plan)),
        "piper_b200_select_plan",
    )
    return PiperAttentionExecutionPlan.from_native(plan)
