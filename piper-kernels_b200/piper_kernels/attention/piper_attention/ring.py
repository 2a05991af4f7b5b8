"""Sequence-sharded ("ring") Piper Attention across the GPUs of one node.

For sequences too long for one GPU's compute budget, rank ``r`` of a process
group holds rows ``[r*n, (r+1)*n)`` of query, key and value (``n`` equal on
every rank) and gets the same rows of the output.  The reference runs on one
GPU only (Piper Kernels 0.2.1, ``attention/piper_attention/dispatch.py:39-83``);
this extends its arithmetic unchanged:

1. each rank sums its K (and, non-causal, V) columns in fp64; one all-reduce of
   the compact ``[2,B,H,D]`` totals gives every rank the sequence means
   (reference.py:46-52), so its INT8 codes and scales are exactly those one
   GPU computes for the same rows (shards start at multiples of 64 rows, so
   no per-64-row K group straddles two ranks);
2. ``world - 1`` ring steps pass each rank's INT8 K/V pack (K codes + scales,
   transposed V codes + per-key vectors) to the next rank with NCCL
   send/recv into a double-buffered receive area, while the attention kernel
   runs over the pack it already holds, carrying every query row's
   online-softmax state (numerator, max, denominator) from one key shard to
   the next; the last step writes the output.

No output gather is needed: each rank owns its query rows.  Causal
attention works with either shard layout (each key range is placed by
``causal_shift``).  With ``layout="contiguous"`` rank r holds rows
[r*n, (r+1)*n) and causal work is unbalanced (the last rank sees every key).
With ``layout="zigzag"`` the sequence is cut into 2*world chunks of n/2 rows
and rank r holds chunks r and 2*world-1-r (use :func:`zigzag_shard`): every
rank then has the same causal work, and each ring step runs the attention for
the (query chunk, key chunk) pairs that are not fully masked.

``ops_factory`` selects the compute backend; the default is the sm_100a
library.  Tests substitute a CPU restatement to exercise this host logic over
``gloo`` ranks.
"""

from __future__ import annotations

import datetime
from typing import Callable, Protocol

import torch
import torch.distributed as dist

from ... import _native
from .._validation import validate_attention_inputs
from . import b200

OPERATOR = "ring_piper_attention"
STATE_LOAD = _native.STATE_LOAD
STATE_STORE = _native.STATE_STORE
SHARD_ALIGNMENT = 64  # rows per K quantization group


class RingStepError(RuntimeError):
    """A ring step's exchange with a neighbour failed or did not finish in time.

    Raised on the ranks that survive a peer which left (raised, exited or
    hung) before finishing the ring.  With ``abort_on_failure`` the group has
    been aborted, so no collective of it is left waiting on the dead peer.
    """


def _abort(group) -> None:
    """Abort the group's communicators, where the backend supports it."""
    pg = group if group is not None else dist.distributed_c10d._get_default_group()
    try:
        pg.abort()
    except (RuntimeError, NotImplementedError, AttributeError):
        pass


class ShardOps(Protocol):
    """Compute steps of one rank's shard (the native backend or a test double)."""

    def column_totals(self) -> torch.Tensor:
        """Launch the shard's column sums; return the fp64 totals to all-reduce in place."""

    def quantize(self, total_keys: int) -> None:
        """Means from the summed totals, then this shard's INT8 codes and scales."""

    def local_pack(self) -> torch.Tensor:
        """This shard's K/V pack (1-D uint8)."""

    def empty_pack(self) -> torch.Tensor:
        """A receive buffer for another rank's pack."""

    def new_state(self) -> torch.Tensor:
        """Per-row softmax state carried between key shards."""

    def attend(self, pack: torch.Tensor, state: torch.Tensor | None, state_mode: int, causal_shift: int,
               out: torch.Tensor, query_range: tuple[int, int] | None = None,
               key_range: tuple[int, int] | None = None, masked: bool | None = None) -> None:
        """Attention of this shard's queries (a row range) over keys in ``pack`` (a key range).

        ``masked=False`` runs a causal problem's launch without the mask (its
        keys all precede its queries).
        """


class NativeShardOps:
    """The sm_100a library on the query's CUDA device, on the current stream."""

    def __init__(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, is_causal: bool,
                 scale: float) -> None:
        if query.device.type != "cuda":
            raise RuntimeError(f"{OPERATOR} requires CUDA tensors on an sm_100 GPU, got {query.device}")
        self.query, self.key, self.value = query, key, value
        self.is_causal = is_causal
        self.scale = scale
        self.prepared: b200.PreparedPiperAttention | None = None

    def column_totals(self) -> torch.Tensor:
        self.prepared = b200.shard_column_sums(self.query, self.key, self.value, self.is_causal)
        return self.prepared.column_totals

    def quantize(self, total_keys: int) -> None:
        assert self.prepared is not None
        b200.shard_prepass(self.query, self.key, self.value, self.prepared, total_keys)

    def local_pack(self) -> torch.Tensor:
        assert self.prepared is not None
        return self.prepared.kv_pack

    def empty_pack(self) -> torch.Tensor:
        return torch.empty_like(self.local_pack())

    def new_state(self) -> torch.Tensor:
        b, h, nq, d = self.query.shape
        return torch.empty(b200.state_bytes(b, h, nq, d) // 4, dtype=torch.float32, device=self.query.device)

    def attend(self, pack, state, state_mode, causal_shift, out, query_range=None, key_range=None,
               masked=None) -> None:
        assert self.prepared is not None
        b200.attention_shard(self.prepared, pack, self.scale, state=state, state_mode=state_mode,
                             causal_shift=causal_shift, out=out, query_range=query_range, key_range=key_range,
                             masked=masked)


def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """Rows of ``x`` (full sequence along ``dim``) that rank ``rank`` holds in the zig-zag layout."""
    n = x.shape[dim]
    if n % (2 * world):
        raise ValueError(f"sequence length {n} does not split into {2 * world} chunks")
    c = n // (2 * world)
    first = x.narrow(dim, rank * c, c)
    second = x.narrow(dim, (2 * world - 1 - rank) * c, c)
    return torch.cat([first, second], dim=dim)


def zigzag_unshard(parts: list[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Reassemble the full sequence from every rank's zig-zag shard (rank order)."""
    world = len(parts)
    c = parts[0].shape[dim] // 2
    chunks: list[torch.Tensor | None] = [None] * (2 * world)
    for r, part in enumerate(parts):
        chunks[r] = part.narrow(dim, 0, c)
        chunks[2 * world - 1 - r] = part.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


def _plan(rank: int, world: int, n: int, is_causal: bool, layout: str):
    """Attention launches per ring step: (query_range, key_range, causal_shift, mode, masked).

    The pack held at step s belongs to rank (rank - s) mod world.  Each query
    range starts its state fresh on its first launch and writes the output on
    its last.  A causal launch whose keys all precede its queries needs no
    mask (masked=False), which lets it use the non-causal kernel path (and its
    split-KV tail).
    """
    steps: list[list[list]] = []
    if layout == "contiguous":
        for s in range(world):
            owner = (rank - s) % world
            shift = (rank - owner) * n if is_causal else 0
            steps.append([[None, None, shift, is_causal and owner >= rank]])
    else:
        c = n // 2
        chunk_of = lambda r, half: r if half == 0 else 2 * world - 1 - r  # noqa: E731
        for s in range(world):
            owner = (rank - s) % world
            step = []
            for qh in (0, 1):
                for kh in (0, 1):
                    iq, ik = chunk_of(rank, qh), chunk_of(owner, kh)
                    if is_causal and ik > iq:
                        continue  # keys entirely after the queries
                    step.append([(qh * c, c), (kh * c, c), (iq - ik) * c if is_causal else 0, is_causal and ik == iq])
            steps.append(step)
    # State modes: per query range, LOAD after its first launch, STORE before its last.
    seen: dict = {}
    total: dict = {}
    for step in steps:
        for launch in step:
            total[launch[0]] = total.get(launch[0], 0) + 1
    for step in steps:
        for launch in step:
            q = launch[0]
            k = seen.get(q, 0)
            mode = (STATE_LOAD if k > 0 else 0) | (STATE_STORE if k + 1 < total[q] else 0)
            seen[q] = k + 1
            launch.insert(3, mode)
    return steps


def _collective_device(group) -> torch.device:
    if dist.get_backend(group) == dist.Backend.NCCL:
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _agree_on_inputs(ok: bool, shape: tuple[int, ...], group) -> tuple[bool, bool]:
    """One small all-reduce: did every rank accept its inputs, with one shape?

    Every rank learns the same answer, so all of them raise together instead
    of some entering the ring's collectives while others have left.
    """
    local = torch.tensor([0 if ok else 1] + [v for s in shape for v in (s, -s)], dtype=torch.int64,
                         device=_collective_device(group))
    seen = local.clone()
    dist.all_reduce(seen, op=dist.ReduceOp.MAX, group=group)
    return bool(seen[0].item() == 0), bool(torch.equal(seen[1:], local[1:]))


def ring_piper_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
    is_causal: bool = False,
    group: dist.ProcessGroup | None = None,
    layout: str = "contiguous",
    ops_factory: Callable[..., ShardOps] | None = None,
    step_timeout: datetime.timedelta | None = None,
    abort_on_failure: bool = False,
) -> torch.Tensor:
    """Piper Attention of a sequence sharded over ``group`` (this rank's rows).

    ``query``/``key``/``value`` are this rank's ``[B, H, n, D]`` shard of the
    sequence; every rank passes the same shape and ``n`` is a multiple of 64
    when there is more than one rank.  Returns this rank's rows of the output,
    equal (up to fp32 rounding in the softmax) to the matching rows of
    ``piper_attention`` on the whole sequence, with identical INT8 codes.
    Without an initialised process group it is ``piper_attention`` on one GPU.
    ``layout`` is "contiguous" or "zigzag" (see the module docstring; with
    "zigzag" the shard length must be a multiple of 128).

    Failure handling: by default each ring step's send/receive is ordered on
    the device stream (no host wait), and a peer that leaves is caught by the
    process group's own timeout.  With ``step_timeout`` the host instead waits
    for every step's exchange, at most that long (the backend's blocking wait
    with a timeout), and raises :class:`RingStepError` naming the step and the
    neighbours when it fails or runs out -- before this rank launches anything
    of the next step.  ``abort_on_failure`` then also aborts the group's
    communicators, so that no collective stays waiting on the lost peer.
    """
    if layout not in ("contiguous", "zigzag"):
        raise ValueError(f"{OPERATOR} layout must be 'contiguous' or 'zigzag', got {layout!r}")
    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    error: Exception | None = None
    try:
        scale = validate_attention_inputs(OPERATOR, query, key, value, scale, is_causal)
        if query.shape[2] != key.shape[2]:
            raise ValueError(f"{OPERATOR} needs equal query and key shard lengths, got "
                             f"{query.shape[2]}/{key.shape[2]}")
    except (ValueError, RuntimeError) as exc:
        error = exc
    if world > 1:
        shape = tuple(query.shape) if query.ndim == 4 else (0, 0, 0, 0)
        all_ok, same_shape = _agree_on_inputs(error is None, shape, group)
        if error is not None:
            raise error
        if not all_ok:
            raise ValueError(f"{OPERATOR}: another rank rejected its inputs")
        if not same_shape:
            raise ValueError(f"{OPERATOR} needs the same [B, H, N, D] shard shape on every rank, got {shape} here")
        align = SHARD_ALIGNMENT * (2 if layout == "zigzag" else 1)
        if query.shape[2] % align:
            raise ValueError(f"{OPERATOR} shards must hold a multiple of {align} rows, got {query.shape[2]}")
    elif error is not None:
        raise error
    n = key.shape[2]
    factory = ops_factory or NativeShardOps
    ops = factory(query, key, value, is_causal, scale)

    totals = ops.column_totals()
    if world > 1:
        dist.all_reduce(totals, op=dist.ReduceOp.SUM, group=group)
    ops.quantize(total_keys=n * world)

    out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    if world == 1:
        ops.attend(ops.local_pack(), None, 0, 0, out)
        return out

    to_rank = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
    from_rank = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world
    plan = _plan(rank, world, n, is_causal, layout)
    state = ops.new_state()
    receive = [ops.empty_pack() for _ in range(2 if world > 2 else 1)]
    held = ops.local_pack()
    for step in range(world):
        last = step + 1 == world
        pending = []
        if not last:
            incoming = receive[step % len(receive)]
            pending = dist.batch_isend_irecv([
                dist.P2POp(dist.isend, held, to_rank, group),
                dist.P2POp(dist.irecv, incoming, from_rank, group),
            ])
        for query_range, key_range, shift, mode, masked in plan[step]:
            ops.attend(held, state, mode, shift if masked else 0, out, query_range=query_range, key_range=key_range,
                       masked=masked)
        for work in pending:
            if step_timeout is None:
                work.wait()
                continue
            try:
                completed = work.wait(step_timeout)
            except Exception as exc:  # the backend's timeout or a broken connection
                if abort_on_failure:
                    _abort(group)
                raise RingStepError(
                    f"{OPERATOR}: rank {rank}, ring step {step}: the K/V exchange with ranks {to_rank}/{from_rank} "
                    f"failed or did not finish within {step_timeout.total_seconds():g} s ({exc})"
                ) from exc
            if completed is False:
                if abort_on_failure:
                    _abort(group)
                raise RingStepError(f"{OPERATOR}: rank {rank}, ring step {step}: the K/V exchange did not complete")
        if not last:
            held = incoming
    return out
