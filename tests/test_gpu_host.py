"""Host-to-host forward (piper_b200_attention_fwd_host) on the GPU (B200 only).

The heads go through the GPU in chunks, with copies overlapping the kernels
of other chunks.  Heads are independent, so the output must equal the
device-memory operator's up to the fp32 rounding of the split-KV tail (a
chunk's last partial wave is split differently from the whole problem's).
"""

from __future__ import annotations

import pytest
import torch
from conftest import require_b200

from piper_kernels import _native, piper_attention
from piper_kernels.attention.piper_attention.b200 import run_piper_attention_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(("b", "h", "n", "d", "dtype", "is_causal"), [
    (1, 1, 300, 64, torch.bfloat16, False),
    (2, 3, 1000, 128, torch.float16, True),
    (1, 40, 2048, 128, torch.bfloat16, False),
    (3, 7, 513, 128, torch.bfloat16, False),
])
def test_host_pipeline_equals_device_operator(b, h, n, d, dtype, is_causal) -> None:
    dev = require_b200()
    g = torch.Generator().manual_seed(b * 100 + h + n)
    q = torch.randn((b, h, n, d), generator=g).to(dtype).pin_memory()
    k = (torch.randn((b, h, n, d), generator=g) + 1).to(dtype).pin_memory()
    v = (torch.randn((b, h, n, d), generator=g) + 0.5).to(dtype).pin_memory()
    with torch.no_grad():
        host = run_piper_attention_host(q, k, v, is_causal=is_causal)
        ref = piper_attention(q.to(dev), k.to(dev), v.to(dev), is_causal=is_causal).cpu()
    assert _native.device_status(0) == 0
    assert host.device.type == "cpu" and host.dtype is dtype
    err = (host.float() - ref.float()).abs()
    assert (err <= 1e-3 + ref.float().abs() / 64).all() and err.mean().item() < 2e-4


def test_host_pipeline_accepts_pageable_memory_and_a_given_output() -> None:
    dev = require_b200()
    g = torch.Generator().manual_seed(3)
    q = torch.randn((1, 5, 256, 128), generator=g).to(torch.float16)
    k = torch.randn((1, 5, 256, 128), generator=g).to(torch.float16)
    out = torch.empty_like(q)
    with torch.no_grad():
        got = run_piper_attention_host(q, k, k, out=out, scale=0.1)
        ref = piper_attention(q.to(dev), k.to(dev), k.to(dev), scale=0.1).cpu()
    assert got is out
    err = (out.float() - ref.float()).abs()
    assert err.max().item() < 0.02 and err.mean().item() < 2e-4


def test_host_pipeline_rejects_device_or_strided_tensors() -> None:
    dev = require_b200()
    q = torch.randn((1, 2, 64, 64), dtype=torch.float16)
    with pytest.raises(ValueError, match="contiguous CPU tensor"):
        run_piper_attention_host(q.to(dev), q.to(dev), q.to(dev))
    t = torch.randn((1, 64, 2, 64), dtype=torch.float16).transpose(1, 2)
    with pytest.raises(ValueError, match="contiguous CPU tensor"):
        run_piper_attention_host(t, t, t)
