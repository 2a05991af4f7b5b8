"""Tensor-core and failure-detection self-tests through the C ABI (B200 only).

* tcgen05.mma kind::i8 through TMA + the UMMA descriptors the attention kernel
  uses: s8 x s8 and u8 x s8 (codes above 127, the case the reference pins in
  tests/triton/test_mixed_int8.py:194-217) must be exact in INT32.
* The bounded-wait path: a CTA waits on an mbarrier that nothing arrives at;
  it must give up within its budget, report the timeout, and leave the
  context usable.
"""

from __future__ import annotations

import ctypes

import pytest
import torch
from conftest import require_b200

from piper_kernels import _native

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_signed", [True, False])
@pytest.mark.parametrize(("m", "n", "k"), [(128, 64, 128), (256, 128, 384)])
def test_int8_tensor_core_gemm_is_exact(a_signed: bool, m: int, n: int, k: int) -> None:
    dev = require_b200()
    g = torch.Generator(device="cpu").manual_seed(m + n + k + int(a_signed))
    if a_signed:
        a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int16).to(torch.int8)
        a_wide = a.to(torch.int64)
    else:
        a_u8 = torch.randint(0, 256, (m, k), generator=g, dtype=torch.int16).to(torch.uint8)
        a = a_u8
        a_wide = a_u8.to(torch.int64)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
    expected = (a_wide @ b.to(torch.int64).T).to(torch.int32)
    a_d, b_d = a.to(dev), b.to(dev)
    c_d = torch.full((m, n), -1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _native.check(
        _native.library().piper_b200_selftest_gemm_i8(
            a_d.data_ptr(), b_d.data_ptr(), c_d.data_ptr(), m, n, k, 1 if a_signed else 0, stream
        ),
        "selftest gemm",
    )
    torch.cuda.synchronize()
    assert _native.device_status(0) == 0
    assert torch.equal(c_d.cpu(), expected)


def test_bounded_wait_gives_up_and_context_survives() -> None:
    dev = require_b200()
    timed_out = ctypes.c_int(-1)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _native.check(
        _native.library().piper_b200_selftest_wait_timeout(20_000_000, ctypes.byref(timed_out), stream),
        "wait self-test",
    )
    assert timed_out.value == 1
    # The context is still healthy: ordinary work runs and the library's own
    # status word was not touched by the probe.
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum().item()) == 1023 * 1024 / 2
    assert _native.device_status(0) == 0
