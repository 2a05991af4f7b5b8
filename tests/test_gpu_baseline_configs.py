"""Parity at the full BASELINE configurations, on the GPU (B200 only).

Each test runs one headline workload at its real size (the seeded global
problem of ``piper_kernels.baseline_configs``) through the public operator,
then checks a seeded sample of (b, h) pairs against the oracle on the very
same tensors:

* INT8 codes and scales of Q, K and V and the K/V sequence means bit for bit;
* the output within the reference's own GPU bounds against its portable path
  (``tests/attention/piper_attention/test_triton.py:139-145``: mean |err|
  < 0.003, max |err| < 0.12), with cosine similarity > 0.9999.

c5 (N = 131072) checks the first 2048 query rows of two heads against all
keys, both for the one-GPU operator and for an 8-rank sequence ring emulated
on one GPU (the shard column sums, the summed totals, the shard prepass and
eight state-carrying launches per rank, as ``ring_piper_attention`` issues
them over NCCL).  Heads are independent (reference.py:46-52) and so are
query rows, so a sample is a full check of the rows it covers.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
from conftest import require_b200

from oracle import oracle
from piper_kernels import _native, piper_attention
from piper_kernels.attention.piper_attention import b200
from piper_kernels.baseline_configs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu

MEAN_ABS_TOL = 0.003  # test_triton.py:144
MAX_ABS_TOL = 0.12  # test_triton.py:145
COSINE_FLOOR = 0.9999
SAMPLE_ROWS = 2048  # c5: query rows per sampled head


def _sample_heads(name: str, count: int = 2) -> list[tuple[int, int]]:
    cfg = CONFIGS[name]
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    picks = torch.randperm(cfg.batch * cfg.heads, generator=g)[:count].tolist()
    return [divmod(u, cfg.heads) for u in sorted(picks)]


def _compare(actual: torch.Tensor, expected: torch.Tensor) -> None:
    a = actual.double().cpu()
    e = expected.double().cpu()
    assert torch.isfinite(a).all()
    err = (a - e).abs()
    assert err.mean().item() < MEAN_ABS_TOL, err.mean().item()
    assert err.max().item() < MAX_ABS_TOL, err.max().item()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), e.flatten(), dim=0).item()
    assert cos > COSINE_FLOOR, cos


def _check_codes(prepared: b200.PreparedPiperAttention, bi: int, hi: int, ref: oracle.Prepared, rows: int) -> None:
    nk = prepared.shape[3]
    exact = {
        "query_int8": (prepared.query_int8[bi, hi, :rows], ref.query_int8[0, 0]),
        "query_scale": (prepared.query_scale[bi, hi, : rows // 32], ref.query_scale[0, 0]),
        "key_int8": (prepared.key_int8[bi, hi], ref.key_int8[0, 0]),
        "key_scale": (prepared.key_scale[bi, hi], ref.key_scale[0, 0]),
        "key_mean": (prepared.key_mean[bi, hi], ref.key_mean[0, 0]),
        "value_int8": (prepared.value_f16_transposed[bi, hi, :, :nk].to(torch.int8).T, ref.value_int8[0, 0]),
        "value_scale": (prepared.value_scale[bi, hi], ref.value_scale[0, 0]),
    }
    if ref.value_mean is not None:
        exact["value_mean"] = (prepared.value_mean[bi, hi], ref.value_mean[0, 0])
    for what, (mine, theirs) in exact.items():
        assert np.array_equal(mine.cpu().numpy(), theirs), f"{what} of head ({bi}, {hi}) differs from the oracle"


@pytest.mark.parametrize("name", ["c2", "c3", "c4"])
def test_full_size_config_matches_oracle(name: str) -> None:
    dev = require_b200()
    cfg = CONFIGS[name]
    q, k, v = make_inputs(name, dev)
    scale = cfg.head_dim**-0.5
    with torch.no_grad():
        out = piper_attention(q, k, v, is_causal=cfg.is_causal)
        prepared = b200.prepare_piper_attention(q, k, v, cfg.is_causal)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    oracle.set_threads(os.cpu_count() or 1)
    for bi, hi in _sample_heads(name):
        head = [t[bi : bi + 1, hi : hi + 1].cpu() for t in (q, k, v)]
        ref_out, ref = oracle.piper_attention(*head, scale, cfg.is_causal)
        _check_codes(prepared, bi, hi, ref, cfg.seq_len)
        _compare(out[bi : bi + 1, hi : hi + 1], torch.from_numpy(ref_out).to(cfg.dtype))


def _emulated_ring(q, k, v, world: int):
    """Every rank's shard of a non-causal sequence ring on one GPU (contiguous shards)."""
    n = q.shape[2] // world
    shards = [tuple(t[:, :, r * n : (r + 1) * n].contiguous() for t in (q, k, v)) for r in range(world)]
    prepared = [b200.shard_column_sums(*sh, False) for sh in shards]
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
            b200.attention_shard(prepared[r], prepared[owner].kv_pack, scale, state=state, state_mode=mode, out=out)
        outs.append(out)
    return outs, prepared


def test_c5_one_gpu_and_eight_rank_ring_match_oracle() -> None:
    dev = require_b200()
    cfg = CONFIGS["c5"]
    q, k, v = make_inputs("c5", dev)
    scale = cfg.head_dim**-0.5
    heads = _sample_heads("c5")
    with torch.no_grad():
        out = piper_attention(q, k, v)
        prepared = b200.prepare_piper_attention(q, k, v, False)
        # The ring over the sampled heads only (the ring's arithmetic is per head).
        sel = [hi for _bi, hi in heads]
        ring_outs, ring_prepared = _emulated_ring(q[:, sel].contiguous(), k[:, sel].contiguous(),
                                                  v[:, sel].contiguous(), world=8)
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    oracle.set_threads(os.cpu_count() or 1)
    for j, (bi, hi) in enumerate(heads):
        qh, kh, vh = (t[bi : bi + 1, hi : hi + 1].cpu() for t in (q, k, v))
        ref_out, ref = oracle.piper_attention(qh[:, :, :SAMPLE_ROWS], kh, vh, scale, False)
        _check_codes(prepared, bi, hi, ref, SAMPLE_ROWS)
        expected = torch.from_numpy(ref_out).to(cfg.dtype)
        _compare(out[bi : bi + 1, hi : hi + 1, :SAMPLE_ROWS], expected)
        # Rank 0 of the ring owns the first 16384 rows; its means are the global ones.
        assert np.array_equal(ring_prepared[0].key_mean[0, j].cpu().numpy(), ref.key_mean[0, 0])
        assert np.array_equal(ring_prepared[0].value_mean[0, j].cpu().numpy(), ref.value_mean[0, 0])
        assert np.array_equal(ring_prepared[0].query_int8[0, j, :SAMPLE_ROWS].cpu().numpy(), ref.query_int8[0, 0])
        _compare(ring_outs[0][:, j : j + 1, :SAMPLE_ROWS], expected)
    # Every ring rank's rows against the one-GPU operator (fp32 re-association only).
    shard = cfg.seq_len // 8
    for r, ring_out in enumerate(ring_outs):
        one = out[:, [hi for _bi, hi in heads], r * shard : (r + 1) * shard]
        err = (ring_out.float() - one.float()).abs()
        assert err.max().item() < 0.02 and err.mean().item() < 2e-4, (r, err.max().item(), err.mean().item())
