"""CPU oracle for the SageAttention2++ forward -- TEST INFRASTRUCTURE ONLY.

Restates, in PyTorch CPU arithmetic, the portable reference of Piper Kernels
0.2.1 with its default ``qk_quantization="per_thread"``:

* ``quantize_query_per_thread`` / ``quantize_key_per_thread`` --
  src/piper_kernels/attention/kernels/qk_quantization/int8/sage/reference.py:23-60
  (one scale for each set of 4 query rows {b, b+8, b+16, b+24} of a 32-row
  block, and for each set of 16 key rows {8a + 2b + c} of a 64-row block);
  K is centred by its sequence mean first (reference.py:88-89);
* ``_quantize_value_per_channel`` -- sage_attention_2pp/reference.py:21-24
  (scale = max_N |v| / 2.25 + 1e-7 per channel, codes FP8 e4m3);
* the 64-key online softmax of sage_attention_2pp/reference.py:63-104: the
  running maximum is shifted by ln(448) so the largest probability of a block
  is 448, probabilities are quantized to FP8 e4m3, the 64-key P.V partial is
  rounded to fp16 and accumulated in fp32 with the per-channel V scale.

Only tests/, __graft_entry__.smoke() and bench.py's CPU leg use it.  Parity
pin: tests/golden/s2pp_*.npz hold outputs of the reference itself
(tests/golden/make_golden_sage2pp.py); tests/test_oracle_sage2pp.py checks
this file against them.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import oracle

QUERY_BLOCK = 32
KEY_BLOCK = 64
PV_BLOCK = 64
EPS = 1e-7
V_FP8_MAX = 2.25
P_FP8_LN_MAX = math.log(448.0)


def _codes(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return torch.round(x / scale).clamp(-127, 127).to(torch.int8)


def quantize_query_per_thread(q: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """INT8 Q codes and a per-row scale (rows r and r+8 of a 32-row block share one)."""
    b, h, n, d = q.shape
    pad = (-n) % QUERY_BLOCK
    x = torch.cat([q.float(), q.new_zeros((b, h, pad, d), dtype=torch.float32)], dim=2)
    blocks = x.view(b, h, -1, 4, 8, d)  # row = 8*a + g
    amax = blocks.abs().amax(dim=(3, 5))  # [b, h, blocks, 8]
    scale = amax / 127 + EPS
    per_row = scale[:, :, :, None, :].expand(b, h, scale.shape[2], 4, 8).reshape(b, h, -1)
    codes = _codes(x, per_row[..., None])
    return codes[:, :, :n], per_row[:, :, :n].contiguous()


def quantize_key_per_thread(k_centered: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """INT8 K codes and a per-key scale (keys 8a + 2g + c of a 64-row block share one)."""
    b, h, n, d = k_centered.shape
    pad = (-n) % KEY_BLOCK
    x = torch.cat([k_centered.float(), k_centered.new_zeros((b, h, pad, d), dtype=torch.float32)], dim=2)
    blocks = x.view(b, h, -1, 8, 4, 2, d)
    amax = blocks.abs().amax(dim=(3, 5, 6))  # [b, h, blocks, 4]
    scale = amax / 127 + EPS
    per_row = scale[:, :, :, None, :, None].expand(b, h, scale.shape[2], 8, 4, 2).reshape(b, h, -1)
    codes = _codes(x, per_row[..., None])
    return codes[:, :, :n], per_row[:, :, :n].contiguous()


def quantize_value_per_channel(v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 e4m3 V codes (as raw bytes) and a per-channel scale [b, h, d]."""
    scale = v.float().abs().amax(dim=2) / V_FP8_MAX + EPS
    codes = (v.float() / scale[:, :, None, :]).to(torch.float8_e4m3fn)
    return codes.view(torch.uint8), scale


def prepare(query, key, value, *, key_mean=None) -> dict:
    """The prepass; ``key_mean`` overrides the (exact fp64) K sequence mean."""
    if key_mean is None:
        key_mean = torch.from_numpy(oracle.sequence_mean(oracle._as_f32(key)))
    km = torch.as_tensor(np.asarray(key_mean, dtype=np.float32))
    q8, qs = quantize_query_per_thread(query)
    k8, ks = quantize_key_per_thread(key.float() - km[:, :, None, :])
    v8, vs = quantize_value_per_channel(value)
    return {"query_int8": q8, "query_scale": qs, "key_int8": k8, "key_scale": ks, "value_fp8": v8,
            "value_scale": vs, "key_mean": km}


def attention_prepared(p: dict, scale: float, is_causal: bool) -> torch.Tensor:
    """The online-softmax recurrence on prepared operands; fp32 [B, H, Nq, D]."""
    q8, qs, k8, ks = p["query_int8"], p["query_scale"], p["key_int8"], p["key_scale"]
    v = p["value_fp8"].view(torch.float8_e4m3fn).float()
    vs = p["value_scale"]
    b, h, nq, d = q8.shape
    nk = k8.shape[2]
    acc = torch.zeros((b, h, nq, d))
    den = torch.zeros((b, h, nq))
    run = torch.full((b, h, nq), -math.inf)
    rows = torch.arange(nq)
    qf = q8.float()
    for start in range(0, nk, PV_BLOCK):
        stop = min(start + PV_BLOCK, nk)
        s = (qf @ k8[:, :, start:stop].float().transpose(-1, -2)) * qs[..., None] * ks[:, :, None, start:stop] * scale
        if is_causal:
            keys = torch.arange(start, stop)
            s = s.masked_fill(keys[None, None, None, :] > rows[None, None, :, None], -math.inf)
        nxt = torch.maximum(run, s.amax(dim=-1) - P_FP8_LN_MAX)
        old = torch.exp(run - nxt)
        prob = torch.nan_to_num(torch.exp(s - nxt[..., None]))
        acc *= old[..., None]
        den = den * old + prob.sum(dim=-1)
        partial = (prob.to(torch.float8_e4m3fn).float() @ v[:, :, start:stop]).to(torch.float16).float()
        acc += partial * vs[:, :, None, :]
        run = nxt
    return acc / den.clamp_min(1e-30)[..., None]


def sage_attention_2pp(query, key, value, scale: float | None = None, is_causal: bool = False, *,
                       key_mean=None) -> tuple[torch.Tensor, dict]:
    """Oracle forward: fp32 output (cast it to the input dtype) and the prepass."""
    scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    p = prepare(query.cpu(), key.cpu(), value.cpu(), key_mean=key_mean)
    return attention_prepared(p, scale, is_causal), p
