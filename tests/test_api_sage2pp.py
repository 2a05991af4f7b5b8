"""SageAttention2++ public API, validation and operator registration -- CPU only.

Mirrors tests/attention/sage_attention_2pp/test_dispatch.py of the reference
(export identity, rejection messages); as for Piper Attention, CPU tensors
raise instead of running a portable fallback.
"""

from __future__ import annotations

import pytest
import torch

import piper_kernels
from piper_kernels import sage_attention_2pp
from piper_kernels._targets import AcceleratorTarget


def _inputs() -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    q = torch.randn(1, 2, 16, 64, dtype=torch.float16)
    return q, torch.randn_like(q), torch.randn_like(q)


def test_package_root_exports_sage_attention_2pp() -> None:
    assert piper_kernels.sage_attention_2pp is sage_attention_2pp
    assert piper_kernels.__all__ == ["piper_attention", "sage_attention_2pp"]


def test_custom_op_is_registered_with_the_reference_schema() -> None:
    schema = str(torch.ops.piper_kernels.sage_attention_2pp.default._schema)
    assert schema.startswith(
        "piper_kernels::sage_attention_2pp(Tensor query, Tensor key, Tensor value, float scale, bool is_causal)"
    )


def test_fake_implementation_gives_contiguous_output_shape() -> None:
    q = torch.empty((2, 3, 40, 64), dtype=torch.float16, device="meta")
    k = torch.empty((2, 3, 70, 64), dtype=torch.float16, device="meta")
    out = torch.ops.piper_kernels.sage_attention_2pp(q, k, k, 0.1, False)
    assert out.shape == q.shape and out.dtype is q.dtype and out.is_contiguous()


def test_cpu_tensors_raise_instead_of_falling_back() -> None:
    q, k, v = _inputs()
    with pytest.raises(RuntimeError, match="SageAttention2\\+\\+'s B200 backend requires CUDA tensors"):
        sage_attention_2pp(q, k, v, scale=0.2)


def test_target_facts_select_sm100_only() -> None:
    assert AcceleratorTarget("cuda", "sm100").supports_tcgen05_fp8
    for arch in ("sm90", "sm89", "sm120", None):
        assert not AcceleratorTarget("cuda", arch).supports_tcgen05_fp8


@pytest.mark.parametrize("dtype", [torch.float32, torch.int8])
def test_rejects_unsupported_dtype(dtype: torch.dtype) -> None:
    q = torch.zeros((1, 1, 8, 64), dtype=dtype)
    with pytest.raises(ValueError, match="SageAttention2\\+\\+.*float16 or bfloat16"):
        sage_attention_2pp(q, q, q)


def test_rejects_mismatched_dtypes() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="share a dtype"):
        sage_attention_2pp(q, k.to(torch.bfloat16), v)


def test_rejects_unsupported_head_dimension() -> None:
    q = torch.randn(1, 1, 8, 32, dtype=torch.float16)
    with pytest.raises(ValueError, match="head dimensions 64 and 128"):
        sage_attention_2pp(q, q, q)


def test_rejects_mismatched_key_value_lengths() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="key/value lengths"):
        sage_attention_2pp(q, k, v[:, :, :-1])


def test_rejects_grouped_query_attention() -> None:
    q = torch.randn(1, 4, 16, 64, dtype=torch.float16)
    k = torch.randn(1, 2, 16, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="equal batch and head dimensions"):
        sage_attention_2pp(q, k, k)


def test_rejects_rectangular_causal_inputs() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="equal query and key lengths"):
        sage_attention_2pp(q[:, :, :-1], k, v, is_causal=True)


@pytest.mark.parametrize(("nq", "nk"), [(0, 8), (8, 0)])
def test_rejects_empty_sequences(nq: int, nk: int) -> None:
    q = torch.empty((1, 1, nq, 64), dtype=torch.float16)
    k = torch.empty((1, 1, nk, 64), dtype=torch.float16)
    with pytest.raises(ValueError, match="does not accept empty"):
        sage_attention_2pp(q, k, k)


def test_rejects_noncontiguous_head_dimension() -> None:
    q = torch.randn(1, 1, 8, 128, dtype=torch.float16)[..., ::2]
    with pytest.raises(ValueError, match="head dimension must be contiguous"):
        sage_attention_2pp(q, q, q)


def test_rejects_autograd() -> None:
    q, k, v = _inputs()
    q.requires_grad_(True)
    with pytest.raises(RuntimeError, match="inference-only"):
        sage_attention_2pp(q, k, v)


@pytest.mark.parametrize("scale", [0.0, -1.0, float("inf"), float("nan")])
def test_rejects_invalid_scale(scale: float) -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="finite and positive"):
        sage_attention_2pp(q, k, v, scale=scale)
