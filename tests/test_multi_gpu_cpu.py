"""Head/batch partition of one problem over ranks, on CPU ``gloo`` ranks.

``piper_attention_multi_gpu`` splits the flattened ``B*H`` pairs of a global
problem into contiguous balanced slices, one per rank, with no collective on
the data path.  Here the one-GPU operator is replaced by the CPU oracle, so
these tests check the host side: which pairs each rank takes, that the
union of the ranks' slices is exactly the one-process result (every (b, h) is
independent, reference.py:46-52), and the optional all-gather.
"""

from __future__ import annotations

import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from piper_kernels.attention.piper_attention.multi_gpu import head_partition, local_heads, piper_attention_multi_gpu


def _oracle_compute(q, k, v, *, scale, is_causal):
    return oracle.piper_attention_torch(q, k, v, scale, is_causal)


def _inputs(b: int, h: int, n: int, d: int):
    g = torch.Generator().manual_seed(b * 100 + h * 10 + n)
    q = torch.randn((b, h, n, d), generator=g).to(torch.float16)
    k = (torch.randn((b, h, n, d), generator=g) + torch.randn((b, h, 1, d), generator=g) * 2).to(torch.float16)
    v = (torch.randn((b, h, n, d), generator=g) + torch.randn((b, h, 1, d), generator=g)).to(torch.float16)
    return q, k, v


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize(("units", "world"), [(40, 8), (40, 3), (128, 8), (5, 8), (1, 1), (48, 5)])
def test_head_partition_is_contiguous_and_balanced(units: int, world: int) -> None:
    parts = head_partition(units, world)
    assert len(parts) == world
    assert sum(c for _f, c in parts) == units
    first = 0
    for f, c in parts:
        assert f == first
        first += c
    counts = [c for _f, c in parts]
    assert max(counts) - min(counts) <= 1 and counts == sorted(counts, reverse=True)


def test_local_heads_crosses_batch_boundaries() -> None:
    x = torch.arange(3 * 4 * 2 * 1).reshape(3, 4, 2, 1)
    pieces = [local_heads(x, r, 5) for r in range(5)]
    assert [p.shape[1] for p in pieces] == [3, 3, 2, 2, 2]
    assert torch.equal(torch.cat(pieces, dim=1).reshape(3, 4, 2, 1), x)


def _worker(rank: int, world: int, port: int, b: int, h: int, is_causal: bool) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        oracle.set_threads(1)
        q, k, v = _inputs(b, h, 96, 64)
        with torch.no_grad():
            mine = piper_attention_multi_gpu(q, k, v, is_causal=is_causal, compute=_oracle_compute)
            full = piper_attention_multi_gpu(q, k, v, is_causal=is_causal, compute=_oracle_compute, gather=True)
        expected = oracle.piper_attention_torch(q, k, v, None, is_causal)
        first, count = head_partition(b * h, world)[rank]
        assert mine.shape == (1, count, 96, 64)
        # Each (b, h) pair is its own problem: the slice equals the one-shot rows exactly.
        assert torch.equal(mine[0], expected.reshape(b * h, 96, 64)[first : first + count])
        assert torch.equal(full, expected)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize(("world", "b", "h", "is_causal"), [(2, 1, 5, False), (3, 2, 4, True), (4, 1, 3, False)])
def test_partition_over_gloo_ranks_equals_one_process(world: int, b: int, h: int, is_causal: bool) -> None:
    mp.spawn(_worker, args=(world, _free_port(), b, h, is_causal), nprocs=world, join=True)


def test_single_process_is_the_whole_problem() -> None:
    q, k, v = _inputs(2, 3, 70, 64)
    with torch.no_grad():
        out = piper_attention_multi_gpu(q, k, v, compute=_oracle_compute)
    assert torch.equal(out, oracle.piper_attention_torch(q, k, v, None, False))
