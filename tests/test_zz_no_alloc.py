"""The allocation-free forward entry point (B200 only; collected last on purpose).

``piper_b200_attention_fwd_no_alloc`` serves callers that cannot allocate
device memory -- a plugin whose host process owns the whole GPU memory budget,
a language binding that can pass tensors in and out but has no device
allocator, a steady-state loop where a possibly synchronising cudaMalloc is not
allowed.  It takes its scratch from a fixed 16 MiB array inside the library.

This file checks it through the C ABI against the ordinary entry point
(``piper_b200_attention_fwd`` with a caller-provided workspace) on two calls
in a row, with different shapes so the second call runs over what the first
left in the shared array, and checks that an oversized problem is refused.
It is named so pytest collects it after every other test file.
"""

from __future__ import annotations

import pytest
import torch
from conftest import require_b200

from piper_kernels import _native

pytestmark = pytest.mark.gpu

MEAN_ABS_TOL = 0.003
MAX_ABS_TOL = 0.12
_DTYPE = {torch.float16: _native.FLOAT16, torch.bfloat16: _native.BFLOAT16}


def _inputs(shape, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=g).to(dtype)
    k = (torch.randn(shape, generator=g) + torch.randn((*shape[:2], 1, shape[3]), generator=g)).to(dtype)
    v = (torch.randn(shape, generator=g) + 0.5).to(dtype)
    return q.to(dev), k.to(dev), v.to(dev)


def _with_workspace(q, k, v, is_causal):
    lib = _native.library()
    b, h, n, d = q.shape
    ws = torch.empty(int(_native.workspace_layout(b, h, n, n, d).total_bytes), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    rc = lib.piper_b200_attention_fwd(
        q.data_ptr(), _native.strides3(q), k.data_ptr(), _native.strides3(k), v.data_ptr(), _native.strides3(v),
        out.data_ptr(), _DTYPE[q.dtype], b, h, n, n, d, d**-0.5, int(is_causal), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream(q.device).cuda_stream,
    )
    _native.check(rc, "piper_b200_attention_fwd")
    return out


def _no_alloc(q, k, v, is_causal):
    lib = _native.library()
    b, h, n, d = q.shape
    out = torch.empty_like(q)
    rc = lib.piper_b200_attention_fwd_no_alloc(
        q.data_ptr(), _native.strides3(q), k.data_ptr(), _native.strides3(k), v.data_ptr(), _native.strides3(v),
        out.data_ptr(), _DTYPE[q.dtype], b, h, n, n, d, d**-0.5, int(is_causal),
        torch.cuda.current_stream(q.device).cuda_stream,
    )
    return rc, out


def test_no_alloc_entry_point_matches_the_workspace_entry_point_twice_in_a_row() -> None:
    dev = require_b200()
    cases = [
        ((1, 4, 1000, 128), torch.bfloat16, False, 11),
        ((2, 2, 777, 64), torch.float16, True, 12),
    ]
    for shape, dtype, is_causal, seed in cases:
        q, k, v = _inputs(shape, dtype, seed, dev)
        expected = _with_workspace(q, k, v, is_causal)
        rc, actual = _no_alloc(q, k, v, is_causal)
        _native.check(rc, "piper_b200_attention_fwd_no_alloc")
        torch.cuda.synchronize()
        assert _native.device_status(0) == 0
        err = (actual.float() - expected.float()).abs()
        assert torch.isfinite(actual).all()
        assert err.mean().item() < MEAN_ABS_TOL
        assert err.max().item() < MAX_ABS_TOL


def test_no_alloc_entry_point_refuses_problems_beyond_its_scratch() -> None:
    dev = require_b200()
    b, h, n, d = 1, 64, 4096, 128
    assert _native.workspace_layout(b, h, n, n, d).total_bytes > _native.NO_ALLOC_WORKSPACE_BYTES
    q = torch.empty((b, h, n, d), dtype=torch.bfloat16, device=dev)
    rc, _ = _no_alloc(q, q, q, False)
    assert rc == _native.ERR_WORKSPACE_TOO_SMALL
    assert "at most 16777216 bytes" in _native.last_error()
