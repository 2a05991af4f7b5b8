"""The kernels' software exp2 against exact 2^x and against the MUFU's ex2.approx (B200 only).

At D=64 the softmax sends one pair of probabilities in eight through an
FMA-pipe exp2 instead of the MUFU unit: a Cody-Waite split x = n + f
(n = round(x) by the 1.5*2^23 add, f in [-1/2, 1/2]), a degree-5 polynomial
for 2^f fitted here for relative error, and 2^n added to the exponent field.
It must be as accurate as the hardware approximation it stands in for, and
-inf (a masked key) must give a probability whose UINT8 code is zero.
"""

from __future__ import annotations

import pytest
import torch
from conftest import require_b200

from piper_kernels import _native

pytestmark = pytest.mark.gpu

REL_BOUND = 2.5e-7  # stated bound of the polynomial over the normal range [-125, 0]


def _run(x: torch.Tensor):
    dev = x.device
    y = torch.empty_like(x)
    hw = torch.empty_like(x)
    _native.check(_native.library().piper_b200_selftest_exp2(x.data_ptr(), y.data_ptr(), hw.data_ptr(), x.numel(),
                                                             torch.cuda.current_stream(dev).cuda_stream),
                  "piper_b200_selftest_exp2")
    torch.cuda.synchronize()
    return y, hw


def test_polynomial_exp2_relative_error_over_the_softmax_range() -> None:
    dev = require_b200()
    g = torch.Generator().manual_seed(2)
    x = torch.cat([torch.linspace(-125.0, 0.0, 4_000_001, dtype=torch.float64).float(),
                   -torch.rand(4_000_000, generator=g) * 125.0,
                   torch.tensor([0.0, -0.5, -1.0, -1.5, -2.5, -0.49999997, -0.50000006, -124.5])])
    y, hw = _run(x.to(dev))
    exact = torch.exp2(x.double())
    rel = (y.cpu().double() - exact).abs() / exact
    rel_hw = (hw.cpu().double() - exact).abs() / exact
    assert rel.max().item() <= REL_BOUND, (rel.max().item(), x[rel.argmax()].item())
    # On a par with the hardware approximation it replaces.
    assert rel.max().item() <= 2.0 * rel_hw.max().item() + 1e-8, (rel.max().item(), rel_hw.max().item())
    assert rel.mean().item() < 1e-7


def test_masked_and_tiny_inputs_give_zero_codes() -> None:
    dev = require_b200()
    x = torch.tensor([-float("inf"), -1e30, -200.0, -126.5, -126.0, -125.5], device=dev)
    y, _ = _run(x)
    y = y.cpu().double()
    assert torch.isfinite(y).all() and (y >= 0).all()
    assert (y <= 2.0**-124).all()  # far below any probability that reaches the denominator's last bit
    assert torch.equal(torch.round(255.0 * y), torch.zeros_like(y))  # UINT8 code 0, as the oracle's exp(-inf) = 0


def test_odd_lengths_and_empty_input() -> None:
    dev = require_b200()
    for n in (0, 1, 3, 257):
        x = -torch.arange(n, dtype=torch.float32, device=dev) / 7.0
        y, _hw = _run(x)
        if n:
            exact = torch.exp2(x.double().cpu())
            assert ((y.cpu().double() - exact).abs() / exact).max().item() <= REL_BOUND
