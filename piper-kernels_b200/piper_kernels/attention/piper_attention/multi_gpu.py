"""Head/batch partition of one Piper Attention problem over the GPUs of one node.

Every (batch, head) pair of Piper Attention is an independent problem: the K
and V sequence means that smooth and centre it reduce over the sequence only
(Piper Kernels 0.2.1, ``attention/piper_attention/reference.py:46-52``;
``kernels/qk_quantization/int8/sage/reference.py:88-89``), and every scale,
code and softmax row stays inside its head.  So the flattened ``B*H`` pairs
split over ranks with no exchange at all: rank ``r`` of ``world`` takes a
contiguous, balanced slice (the first ``B*H % world`` ranks one pair more)
and runs the one-GPU operator on it.  The reference has no multi-GPU entry
point; this is the partition its shapes allow.

No collective is on the data path.  ``gather=True`` assembles the full output
on every rank with one all-gather afterwards, for validation or for callers
that need it.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .._validation import validate_attention_inputs

OPERATOR = "piper_attention_multi_gpu"


def head_partition(units: int, world: int) -> list[tuple[int, int]]:
    """(first, count) of the contiguous ``B*H`` slice each rank takes."""
    if units < 0 or world < 1:
        raise ValueError("units must be non-negative and world positive")
    base, extra = divmod(units, world)
    slices, first = [], 0
    for r in range(world):
        count = base + (1 if r < extra else 0)
        slices.append((first, count))
        first += count
    return slices


def local_heads(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank ``rank``'s slice of the flattened ``B*H`` pairs of ``x`` as a ``[1, count, N, D]`` view."""
    b, h, n, d = x.shape
    first, count = head_partition(b * h, world)[rank]
    return x.reshape(b * h, n, d)[first : first + count].unsqueeze(0)


def piper_attention_multi_gpu(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
    is_causal: bool = False,
    group: dist.ProcessGroup | None = None,
    gather: bool = False,
    compute: Callable[..., torch.Tensor] | None = None,
) -> torch.Tensor:
    """Piper Attention of the global ``[B, H, N, D]`` problem, split by ``B*H`` over ``group``.

    Every rank passes the same global tensors (each on its own device).  The
    rank computes only its slice (:func:`local_heads`) and returns that
    slice's output as ``[1, count, Nq, D]``, or, with ``gather=True``, the
    whole ``[B, H, Nq, D]`` output (one all-gather).  Without an initialised
    process group it is ``piper_attention`` on the whole problem.  ``compute``
    replaces the one-GPU operator (tests pass a CPU restatement); it takes
    ``(query, key, value, scale=..., is_causal=...)``.
    """
    scale = validate_attention_inputs(OPERATOR, query, key, value, scale, is_causal)
    if compute is None:
        from .dispatch import piper_attention as compute
    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    b, h, nq, d = query.shape
    q, k, v = (local_heads(t, rank, world) for t in (query, key, value))
    if q.shape[1] > 0:
        out_local = compute(q, k, v, scale=scale, is_causal=is_causal)
    else:
        out_local = torch.empty((1, 0, nq, d), dtype=query.dtype, device=query.device)
    if not gather or world == 1:
        return out_local.reshape(b, h, nq, d) if world == 1 else out_local
    # all_gather wants equal pieces: pad every slice to the largest.
    parts = head_partition(b * h, world)
    widest = max(count for _first, count in parts)
    piece = torch.zeros((widest, nq, d), dtype=query.dtype, device=out_local.device)
    piece[: out_local.shape[1]] = out_local[0]
    gathered = [torch.empty_like(piece) for _ in range(world)]
    dist.all_gather(gathered, piece, group=group)
    full = torch.cat([gathered[r][:count] for r, (_first, count) in enumerate(parts)])
    return full.reshape(b, h, nq, d)
