"""Host logic of the sequence-sharded ring on CPU: ``gloo`` ranks, oracle compute.

The ring driver (``ring_piper_attention``) takes its compute steps from a
``ShardOps`` object; here that object is the CPU oracle (a test double that
stands where the sm_100a library does on a GPU), so these tests check what the
host side decides: the all-reduced column totals and the means made from
them, which pack each rank holds at each step, the double-buffered exchange,
the state modes and the causal shifts.  Each rank's rows must match the
one-shot oracle on the whole sequence (codes bit for bit, outputs to fp32
rounding), for 2, 3 and 4 ranks, causal and not.
"""

from __future__ import annotations

import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from piper_kernels.attention.piper_attention.ring import _plan, ring_piper_attention, zigzag_shard, zigzag_unshard


class OracleShardOps:
    """``ShardOps`` over the CPU oracle; packs are serialised to uint8 tensors."""

    instances: list["OracleShardOps"] = []

    def __init__(self, query, key, value, is_causal, scale):
        self.q, self.k, self.v = query, key, value
        self.is_causal = is_causal
        self.scale = scale
        self.b, self.h, self.n, self.d = query.shape
        self.prepared = None
        OracleShardOps.instances.append(self)

    def column_totals(self):
        # The driver all-reduces this tensor in place; quantize reads it back.
        kt = self.k.double().sum(dim=2)
        vt = torch.zeros_like(kt) if self.is_causal else self.v.double().sum(dim=2)
        self.totals = torch.stack([kt, vt])
        return self.totals

    def quantize(self, total_keys):
        km = (self.totals[0].numpy() / float(total_keys)).astype(np.float32)
        vm = None if self.is_causal else (self.totals[1].numpy() / float(total_keys)).astype(np.float32)
        self.prepared = oracle.prepare(self.q, self.k, self.v, self.is_causal, key_mean=km, value_mean=vm)

    def _pieces(self):
        p = self.prepared
        return [p.key_int8, p.key_scale, p.value_int8, p.value_scale]

    def local_pack(self):
        raw = b"".join(np.ascontiguousarray(a).tobytes() for a in self._pieces())
        return torch.frombuffer(bytearray(raw), dtype=torch.uint8)

    def empty_pack(self):
        return torch.empty_like(self.local_pack())

    def _unpack(self, pack):
        data = pack.numpy().tobytes()
        out, at = [], 0
        for ref in self._pieces():
            nbytes = ref.nbytes
            out.append(np.frombuffer(data[at : at + nbytes], dtype=ref.dtype).reshape(ref.shape))
            at += nbytes
        assert at == len(data)
        k8, ks, v8, vs = out
        return SimpleNamespace(key_int8=k8, key_scale=ks, value_int8=v8, value_scale=vs)

    def new_state(self):
        return torch.zeros(self.b * self.h * self.n * (self.d + 2), dtype=torch.float32)

    def attend(self, pack, state, state_mode, causal_shift, out, query_range=None, key_range=None, masked=None):
        q0, qn = query_range if query_range is not None else (0, self.n)
        k0, kn = key_range if key_range is not None else (0, self.n)
        assert q0 % 64 == 0 and k0 % 64 == 0
        keys = self._unpack(pack)
        p = self.prepared
        query_side = SimpleNamespace(
            query_int8=np.ascontiguousarray(p.query_int8[:, :, q0 : q0 + qn]),
            query_scale=np.ascontiguousarray(p.query_scale[:, :, q0 // 32 : (q0 + qn + 31) // 32]),
            value_mean=p.value_mean,
        )
        key_side = SimpleNamespace(
            key_int8=np.ascontiguousarray(keys.key_int8[:, :, k0 : k0 + kn]),
            key_scale=np.ascontiguousarray(keys.key_scale[:, :, k0 // 64 : (k0 + kn + 63) // 64]),
            value_int8=np.ascontiguousarray(keys.value_int8[:, :, k0 : k0 + kn]),
            value_scale=np.ascontiguousarray(keys.value_scale[:, :, k0 : k0 + kn]),
        )
        pair = None
        if state is not None:
            cut = self.b * self.h * self.n * self.d
            arr = state.numpy()
            so = arr[:cut].reshape(self.b, self.h, self.n, self.d)
            sml = arr[cut:].reshape(self.b, self.h, self.n, 2)
            pair = (np.ascontiguousarray(so[:, :, q0 : q0 + qn]), np.ascontiguousarray(sml[:, :, q0 : q0 + qn]))
        causal = self.is_causal if masked is None else (self.is_causal and masked)
        result = oracle.attention_shard(query_side, key_side, self.scale, causal, causal_shift=causal_shift,
                                        state=pair, state_mode=state_mode)
        if pair is not None and state_mode & oracle.STATE_STORE:
            so[:, :, q0 : q0 + qn] = pair[0]
            sml[:, :, q0 : q0 + qn] = pair[1]
        if result is not None:
            out[:, :, q0 : q0 + qn] = torch.from_numpy(result).to(out.dtype)


def _inputs(n_total: int, d: int, dtype):
    g = torch.Generator().manual_seed(n_total + d)
    q = torch.randn((1, 2, n_total, d), generator=g).to(dtype)
    k = (torch.randn((1, 2, n_total, d), generator=g) + torch.randn((1, 2, 1, d), generator=g) * 2).to(dtype)
    v = (torch.randn((1, 2, n_total, d), generator=g) + torch.randn((1, 2, 1, d), generator=g)).to(dtype)
    return q, k, v


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n_shard: int, d: int, is_causal: bool, layout: str = "contiguous") -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        oracle.set_threads(1)
        q, k, v = _inputs(n_shard * world, d, torch.float16)
        if layout == "zigzag":
            def part(x):
                return zigzag_shard(x, rank, world) if torch.is_tensor(x) else \
                    zigzag_shard(torch.from_numpy(np.ascontiguousarray(x)), rank, world).numpy()
            with torch.no_grad():
                out = ring_piper_attention(part(q), part(k), part(v), is_causal=is_causal, layout="zigzag",
                                           ops_factory=OracleShardOps)
            full, prepared = oracle.piper_attention(q, k, v, None, is_causal)
            mine = OracleShardOps.instances[-1].prepared
            assert np.array_equal(mine.key_int8, part(prepared.key_int8))
            assert np.array_equal(mine.value_int8, part(prepared.value_int8))
            assert np.array_equal(mine.query_int8, part(prepared.query_int8))
            expected = part(torch.from_numpy(full)).to(out.dtype).float()
            err = (out.float() - expected).abs()
            assert err.max().item() <= 2e-3 * max(1.0, expected.abs().max().item()), err.max().item()
            assert (err > 0).float().mean().item() < 1e-3
            return
        rows = slice(rank * n_shard, (rank + 1) * n_shard)
        with torch.no_grad():
            out = ring_piper_attention(q[:, :, rows], k[:, :, rows], v[:, :, rows], is_causal=is_causal,
                                       ops_factory=OracleShardOps)
        full, prepared = oracle.piper_attention(q, k, v, None, is_causal)
        mine = OracleShardOps.instances[-1].prepared
        assert np.array_equal(mine.key_mean, prepared.key_mean)
        assert np.array_equal(mine.query_int8, prepared.query_int8[:, :, rows])
        assert np.array_equal(mine.key_int8, prepared.key_int8[:, :, rows])
        assert np.array_equal(mine.key_scale, prepared.key_scale[:, :, rank * n_shard // 64 : (rank + 1) * n_shard // 64])
        assert np.array_equal(mine.value_int8, prepared.value_int8[:, :, rows])
        assert np.array_equal(mine.value_scale, prepared.value_scale[:, :, rows])
        expected = torch.from_numpy(full[:, :, rows]).to(out.dtype).float()
        err = (out.float() - expected).abs()
        # The re-associated recurrence differs from the one-shot one by fp32
        # rounding only: after the cast to fp16 at most one ulp, rarely.
        assert err.max().item() <= 2e-3 * max(1.0, expected.abs().max().item()), err.max().item()
        assert (err > 0).float().mean().item() < 1e-3
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("is_causal", [False, True])
def test_ring_matches_one_shot_oracle(world: int, is_causal: bool) -> None:
    mp.spawn(_worker, args=(world, _free_port(), 128, 64, is_causal), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("is_causal", [True, False])
def test_zigzag_ring_matches_one_shot_oracle(world: int, is_causal: bool) -> None:
    mp.spawn(_worker, args=(world, _free_port(), 128, 64, is_causal, "zigzag"), nprocs=world, join=True)


def test_zigzag_plan_balances_causal_work() -> None:
    # Work per rank in block-pair units: a full chunk pair counts 1, a
    # diagonal pair 1/2.  Contiguous shards give rank r work r + 1/2.
    for world in (2, 4, 8):
        works = []
        for r in range(world):
            w = 0.0
            for step in _plan(r, world, 256, True, "zigzag"):
                for _q, _k, shift, _mode, masked in step:
                    assert masked == (shift == 0)  # only diagonal pairs need the mask
                    w += 0.5 if shift == 0 else 1.0
            works.append(w)
        assert len(set(works)) == 1, works
        # (2*world)^2 / 2 chunk pairs are visible in all, spread evenly.
        assert works[0] == 2.0 * world


def _mismatch_worker(rank: int, world: int, port: int, case: str) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        n = 128
        if case == "shape" and rank == 1:
            n = 192
        if case == "alignment":
            n = 100
        q, k, v = _inputs(n, 64, torch.float16)
        if case == "dtype" and rank == 0:
            v = v.to(torch.bfloat16)
        expected = {
            "shape": "same \\[B, H, N, D\\] shard shape",
            "alignment": "multiple of 64 rows",
            "dtype": "share a dtype" if rank == 0 else "another rank rejected",
        }[case]
        with torch.no_grad(), pytest.raises(ValueError, match=expected):
            ring_piper_attention(q, k, v, ops_factory=OracleShardOps)
        # Every rank left together: the group still works.
        t = torch.ones(1)
        dist.all_reduce(t)
        assert t.item() == world
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["shape", "alignment", "dtype"])
def test_ring_rejects_inputs_on_every_rank(case: str) -> None:
    mp.spawn(_mismatch_worker, args=(2, _free_port(), case), nprocs=2, join=True)


def test_zigzag_shard_round_trip() -> None:
    x = torch.arange(2 * 3 * 24 * 4).reshape(2, 3, 24, 4)
    parts = [zigzag_shard(x, r, 3) for r in range(3)]
    assert torch.equal(parts[0][:, :, :4], x[:, :, 0:4]) and torch.equal(parts[0][:, :, 4:], x[:, :, 20:24])
    assert torch.equal(zigzag_unshard(parts), x)


def test_single_process_ring_is_the_one_shot_operator() -> None:
    q, k, v = _inputs(200, 64, torch.bfloat16)
    with torch.no_grad():
        out = ring_piper_attention(q, k, v, is_causal=True, ops_factory=OracleShardOps)
    expected = oracle.piper_attention_torch(q, k, v, None, True)
    assert torch.equal(out, expected)


class SimulatedRankFailure(RuntimeError):
    """The host-made failure of the leaving rank."""


class FailingShardOps(OracleShardOps):
    """Oracle ops that fail on one rank: before the ring ("quantize") or in its second step ("attend")."""

    fail_rank = -1
    fail_at = ""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.attends = 0

    def quantize(self, total_keys):
        if dist.get_rank() == self.fail_rank and self.fail_at == "quantize":
            raise SimulatedRankFailure("rank leaves after the totals all-reduce")
        super().quantize(total_keys)

    def attend(self, *args, **kwargs):
        self.attends += 1
        if dist.get_rank() == self.fail_rank and self.fail_at == "attend" and self.attends == 1:
            raise SimulatedRankFailure("rank leaves in ring step 0, before forwarding any pack")
        super().attend(*args, **kwargs)


def _leaving_worker(rank: int, world: int, port: int, fail_at: str, then: str, results) -> None:
    import datetime
    import time

    from piper_kernels.attention.piper_attention.ring import RingStepError

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    oracle.set_threads(1)
    FailingShardOps.fail_rank, FailingShardOps.fail_at = 1, fail_at
    q, k, v = _inputs(128 * world, 64, torch.float16)
    rows = slice(rank * 128, (rank + 1) * 128)
    t0 = time.monotonic()
    try:
        with torch.no_grad():
            out = ring_piper_attention(q[:, :, rows], k[:, :, rows], v[:, :, rows], ops_factory=FailingShardOps,
                                       step_timeout=datetime.timedelta(seconds=3), abort_on_failure=True)
        # A survivor may finish when every pack it needs had already left the
        # departed rank; its rows must then be right.
        expected = oracle.piper_attention_torch(q, k, v, None, False)[:, :, rows]
        results[rank] = ("finished" if torch.equal(out, expected) else "wrong", time.monotonic() - t0)
    except SimulatedRankFailure:
        results[rank] = ("left", time.monotonic() - t0)
        if then == "hang":
            time.sleep(12)  # alive but silent: the others must give up on their own clock
        return  # leave without tearing the group down
    except RingStepError:
        results[rank] = ("raised", time.monotonic() - t0)
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_at", ["quantize", "attend"])
@pytest.mark.parametrize("then", ["exit", "hang"])
def test_surviving_ranks_raise_when_a_rank_leaves_the_ring(fail_at: str, then: str) -> None:
    # A rank that fails on the host between ring steps (SURVEY: failure
    # detection without a GPU fault): every other rank raises RingStepError
    # within the step timeout instead of waiting forever.
    world = 3
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        procs = [ctx.Process(target=_leaving_worker, args=(r, world, _free_port() if r < 0 else port, fail_at, then,
                                                           results))
                 for port in [_free_port()] for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=90)
        alive = [p.pid for p in procs if p.is_alive()]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert not alive, f"ranks still running: {alive}"
        outcome = dict(results)
    assert outcome[1][0] == "left"
    survivors = [outcome[r] for r in (0, 2)]
    assert all(status in ("raised", "finished") and seconds < 30 for status, seconds in survivors), outcome
    # Without rank 1 after the totals, nobody gets its pack; failing in step 0
    # it forwards nothing, so at least its successor cannot finish.
    if fail_at == "quantize":
        assert all(status == "raised" for status, _ in survivors), outcome
    assert outcome[2][0] == "raised", outcome
