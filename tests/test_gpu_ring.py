"""Sequence-sharded kernels on the GPU (B200 only).

One GPU emulates ``world`` ranks by calling the shard entry points of the C
ABI in the ring's order: fp64 column sums per shard, summed totals, the shard
prepass, then attention over each key shard with the softmax state carried
between launches.  The codes must be bit-identical to the one-shot prepass,
and the output must match the one-shot kernel (the recurrence re-associated
over shards: fp32 rounding only) and the oracle (the usual tolerances).  With
two or more GPUs the real NCCL ring runs under torchrun (``ring_worker.py``).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import require_b200

from oracle import oracle
from piper_kernels import _native, piper_attention
from piper_kernels.attention.piper_attention import b200, ring_piper_attention
from piper_kernels.attention.piper_attention.ring import _plan, zigzag_shard

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def _inputs(n_total: int, d: int, dtype, seed: int):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((2, 2, n_total, d), generator=g).to(dtype)
    k = (torch.randn((2, 2, n_total, d), generator=g) + torch.randn((2, 2, 1, d), generator=g) * 2).to(dtype)
    v = (torch.randn((2, 2, n_total, d), generator=g) + torch.randn((2, 2, 1, d), generator=g)).to(dtype)
    return q, k, v


def _emulated_ring(q, k, v, world: int, is_causal: bool):
    """All ranks' shards on one GPU; returns (outputs per rank, prepared per rank)."""
    n = q.shape[2] // world
    rows = [slice(r * n, (r + 1) * n) for r in range(world)]
    shards = [(q[:, :, s].contiguous(), k[:, :, s].contiguous(), v[:, :, s].contiguous()) for s in rows]
    prepared = [b200.shard_column_sums(*sh, is_causal) for sh in shards]
    totals = sum(p.column_totals for p in prepared)
    for p, sh in zip(prepared, shards):
        p.column_totals.copy_(totals)
        b200.shard_prepass(*sh, p, total_keys=n * world)
    scale = q.shape[-1] ** -0.5
    outs = []
    for r in range(world):
        b_, h_, _, d_ = shards[r][0].shape
        state = torch.empty(b200.state_bytes(b_, h_, n, d_) // 4, dtype=torch.float32, device=q.device)
        out = torch.empty_like(shards[r][0])
        for step in range(world):
            owner = (r - step) % world
            mode = (_native.STATE_LOAD if step else 0) | (0 if step + 1 == world else _native.STATE_STORE)
            b200.attention_shard(prepared[r], prepared[owner].kv_pack, scale, state=state, state_mode=mode,
                                 causal_shift=(r - owner) * n if is_causal else 0, out=out)
        outs.append(out)
    return outs, prepared


def _emulated_zigzag_ring(q, k, v, world: int, is_causal: bool):
    """The zig-zag layout through the range entry point, every rank on one GPU."""
    shards = [tuple(zigzag_shard(t, r, world).contiguous() for t in (q, k, v)) for r in range(world)]
    n = shards[0][0].shape[2]
    prepared = [b200.shard_column_sums(*sh, is_causal) for sh in shards]
    totals = sum(p.column_totals for p in prepared)
    for p, sh in zip(prepared, shards):
        p.column_totals.copy_(totals)
        b200.shard_prepass(*sh, p, total_keys=n * world)
    scale = q.shape[-1] ** -0.5
    outs = []
    for r in range(world):
        b_, h_, _, d_ = shards[r][0].shape
        state = torch.empty(b200.state_bytes(b_, h_, n, d_) // 4, dtype=torch.float32, device=q.device)
        out = torch.empty_like(shards[r][0])
        for step, launches in enumerate(_plan(r, world, n, is_causal, "zigzag")):
            owner = (r - step) % world
            for q_range, k_range, shift, mode, masked in launches:
                b200.attention_shard(prepared[r], prepared[owner].kv_pack, scale, state=state, state_mode=mode,
                                     causal_shift=shift, out=out, query_range=q_range, key_range=k_range,
                                     masked=masked)
        outs.append(out)
    return outs


@pytest.mark.parametrize(("world", "n", "dtype", "is_causal"), [
    (2, 512, torch.bfloat16, True),
    (4, 256, torch.float16, True),
    (3, 384, torch.bfloat16, False),
])
def test_zigzag_ring_matches_one_shot(world, n, dtype, is_causal) -> None:
    dev = require_b200()
    q, k, v = _inputs(world * n, 128, dtype, seed=world * 77 + n)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    with torch.no_grad():
        outs = _emulated_zigzag_ring(qd, kd, vd, world, is_causal)
        shot = piper_attention(qd, kd, vd, is_causal=is_causal)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    expected = oracle.piper_attention_torch(q, k, v, 128**-0.5, is_causal).float()
    for r, out in enumerate(outs):
        err = (out.float() - zigzag_shard(shot, r, world).float()).abs()
        assert err.max().item() < 0.02 and err.mean().item() < 2e-4, (r, err.max().item(), err.mean().item())
        # Against the oracle on the same tensors: the reference's GPU bounds.
        ref_err = (out.float().cpu() - zigzag_shard(expected, r, world)).abs()
        assert ref_err.mean().item() < 0.003 and ref_err.max().item() < 0.12, (r, ref_err.max().item())


def test_key_range_split_with_state_equals_one_launch() -> None:
    # One shard's keys split into three ranges (split-KV), state carried.
    dev = require_b200()
    q, k, v = _inputs(1024, 128, torch.bfloat16, seed=11)
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    with torch.no_grad():
        p = b200.prepare_piper_attention(qd, kd, vd, False)
        whole = b200.launch_piper_attention(p, 128**-0.5)
        state = torch.empty(b200.state_bytes(2, 2, 1024, 128) // 4, dtype=torch.float32, device=dev)
        out = torch.empty_like(qd)
        for i, (k0, kn) in enumerate([(0, 320), (320, 448), (768, 256)]):
            mode = (_native.STATE_LOAD if i else 0) | (_native.STATE_STORE if i < 2 else 0)
            b200.attention_shard(p, p.kv_pack, 128**-0.5, state=state, state_mode=mode, out=out,
                                 key_range=(k0, kn), query_range=(0, 1024))
        # Rows in two ranges as well: the second half of the rows only.
        half = torch.zeros_like(qd)
        b200.attention_shard(p, p.kv_pack, 128**-0.5, out=half, query_range=(512, 512))
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    err = (out.float() - whole.float()).abs()
    assert err.max().item() < 0.02 and err.mean().item() < 2e-4
    e2 = (half[:, :, 512:].float() - whole[:, :, 512:].float()).abs()
    assert e2.max().item() < 0.02 and e2.mean().item() < 2e-4
    assert not half[:, :, :512].any()


@pytest.mark.parametrize(("world", "n", "d", "dtype", "is_causal"), [
    (2, 1024, 128, torch.bfloat16, False),
    (3, 320, 64, torch.float16, False),
    (4, 512, 128, torch.float16, True),
    (2, 2048, 64, torch.bfloat16, True),
    (8, 256, 128, torch.bfloat16, False),
])
def test_sharded_kernels_match_one_shot(world, n, d, dtype, is_causal) -> None:
    dev = require_b200()
    q, k, v = _inputs(world * n, d, dtype, seed=world * 1000 + n)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    with torch.no_grad():
        outs, prepared = _emulated_ring(qd, kd, vd, world, is_causal)
        one = b200.prepare_piper_attention(qd, kd, vd, is_causal)
        one_out = b200.launch_piper_attention(one, d**-0.5)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    for r, p in enumerate(prepared):
        rows = slice(r * n, (r + 1) * n)
        assert torch.equal(p.key_mean, one.key_mean)
        assert torch.equal(p.value_mean, one.value_mean)
        assert torch.equal(p.query_int8, one.query_int8[:, :, rows])
        assert torch.equal(p.key_int8, one.key_int8[:, :, rows])
        assert torch.equal(p.value_int8, one.value_int8[:, :, rows])
        assert torch.equal(p.query_scale, one.query_scale[:, :, r * n // 32 : (r + 1) * n // 32])
        assert torch.equal(p.key_scale, one.key_scale[:, :, r * n // 64 : (r + 1) * n // 64])
        assert torch.equal(p.value_scale, one.value_scale[:, :, rows])
    ring = torch.cat(outs, dim=2).float().cpu()
    shot = one_out.float().cpu()
    err = (ring - shot).abs()
    # Same codes and weights; the re-associated fp32 recurrence moves an output
    # by at most an ulp or two of the output dtype.
    assert err.max().item() < 0.02, err.max().item()
    assert err.mean().item() < 2e-4, err.mean().item()
    expected = oracle.piper_attention_torch(q, k, v, d**-0.5, is_causal).float()
    e2 = (ring - expected).abs()
    assert e2.mean().item() < 0.003 and e2.max().item() < 0.12
    cos = torch.nn.functional.cosine_similarity(ring.double().flatten(), expected.double().flatten(), dim=0).item()
    assert cos > 0.9999


def test_sharded_kernels_restore_constant_value_exactly() -> None:
    dev = require_b200()
    g = torch.Generator().manual_seed(71)
    q = torch.randn((1, 2, 1024, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 2, 1024, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((1, 2, 1, 128), generator=g).to(torch.bfloat16).expand_as(q).contiguous()
    with torch.no_grad():
        outs, _ = _emulated_ring(q.to(dev), k.to(dev), v.to(dev), 4, False)
    torch.testing.assert_close(torch.cat(outs, dim=2).cpu(), v, atol=0.0, rtol=0.0)


def test_fully_masked_key_shard_passes_state_through() -> None:
    # A causal key shard entirely after the query shard: the launch must leave
    # the carried state unchanged (and write the output from it when last).
    dev = require_b200()
    q, k, v = _inputs(512, 64, torch.float16, seed=5)
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    with torch.no_grad():
        first = b200.shard_column_sums(qd[:, :, :256], kd[:, :, :256], vd[:, :, :256], True)
        second = b200.shard_column_sums(qd[:, :, 256:], kd[:, :, 256:], vd[:, :, 256:], True)
        totals = first.column_totals + second.column_totals
        for p, s in ((first, slice(0, 256)), (second, slice(256, 512))):
            p.column_totals.copy_(totals)
            b200.shard_prepass(qd[:, :, s], kd[:, :, s], vd[:, :, s], p, total_keys=512)
        state = torch.empty(b200.state_bytes(2, 2, 256, 64) // 4, dtype=torch.float32, device=dev)
        b200.attention_shard(first, first.kv_pack, 0.125, state=state, state_mode=_native.STATE_STORE)
        kept = state.clone()
        b200.attention_shard(first, second.kv_pack, 0.125, state=state,
                             state_mode=_native.STATE_LOAD | _native.STATE_STORE, causal_shift=-256)
        assert torch.equal(state, kept)
        out = b200.attention_shard(first, second.kv_pack, 0.125, state=state, state_mode=_native.STATE_LOAD,
                                   causal_shift=-256)
        direct = b200.attention_shard(first, first.kv_pack, 0.125)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    assert (out.float() - direct.float()).abs().max().item() < 2e-3


def test_single_process_ring_equals_piper_attention() -> None:
    dev = require_b200()
    q, k, v = _inputs(1000, 128, torch.bfloat16, seed=9)
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    with torch.no_grad():
        ring = ring_piper_attention(qd, kd, vd)
        shot = piper_attention(qd, kd, vd)
    assert torch.equal(ring, shot)


def test_shard_entry_points_reject_bad_arguments() -> None:
    dev = require_b200()
    q, k, v = _inputs(128, 64, torch.float16, seed=3)
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    p = b200.shard_column_sums(qd, kd, vd, False)
    with pytest.raises(ValueError, match="total_keys"):
        b200.shard_prepass(qd, kd, vd, p, total_keys=64)
    b200.shard_prepass(qd, kd, vd, p, total_keys=128)
    with pytest.raises(ValueError, match="causal_shift"):
        b200.attention_shard(p, p.kv_pack, 0.1, causal_shift=64)
    with pytest.raises(ValueError, match="NULL state"):
        b200.attention_shard(p, p.kv_pack, 0.1, state_mode=_native.STATE_LOAD)
    with pytest.raises(ValueError, match="256-byte aligned"):
        b200.attention_shard(p, p.kv_pack[16:], 0.1)
    with pytest.raises(ValueError, match="multiples of 64"):
        b200.attention_shard(p, p.kv_pack, 0.1, key_range=(32, 64))
    with pytest.raises(ValueError, match="outside the problem"):
        b200.attention_shard(p, p.kv_pack, 0.1, query_range=(64, 128))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="the NCCL ring needs two GPUs")
def test_nccl_ring_on_two_gpus() -> None:
    require_b200()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29531", str(REPO / "tests" / "ring_worker.py")]
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert proc.stdout.count("RING_OK") == 2, proc.stdout[-3000:]
