"""Public API, validation and operator registration -- CPU only.

Mirrors tests/attention/piper_attention/test_dispatch.py of the reference
(export identity, rejection messages) and documents the one deliberate
difference: no portable fallback, so CPU tensors raise instead of running.
"""

from __future__ import annotations

import pytest
import torch

import piper_kernels
from piper_kernels import piper_attention
from piper_kernels._targets import AcceleratorTarget


def _inputs() -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    q = torch.randn(1, 2, 16, 64, dtype=torch.float16)
    return q, torch.randn_like(q), torch.randn_like(q)


def test_package_root_exports_piper_attention() -> None:
    assert piper_kernels.piper_attention is piper_attention
    assert "piper_attention" in piper_kernels.__all__


def test_custom_op_is_registered_with_the_reference_schema() -> None:
    op = torch.ops.piper_kernels.piper_attention
    schema = str(op.default._schema)
    assert schema.startswith("piper_kernels::piper_attention(Tensor query, Tensor key, Tensor value, float scale, bool is_causal)")


def test_fake_implementation_gives_contiguous_output_shape() -> None:
    q = torch.empty((2, 3, 40, 128), dtype=torch.bfloat16, device="meta").transpose(1, 2).transpose(1, 2)
    k = torch.empty((2, 3, 50, 128), dtype=torch.bfloat16, device="meta")
    out = torch.ops.piper_kernels.piper_attention(q, k, k, 0.1, False)
    assert out.shape == q.shape and out.dtype is q.dtype and out.is_contiguous()


def test_cpu_tensors_raise_instead_of_falling_back() -> None:
    # Deliberate difference from the reference (test_dispatch.py:23-34 runs the
    # portable path on CPU): the B200 package never computes off the GPU.
    q, k, v = _inputs()
    with pytest.raises(RuntimeError, match="requires CUDA tensors on an sm_100 GPU"):
        piper_attention(q, k, v, scale=0.2)


def test_target_facts_select_sm100_only() -> None:
    assert AcceleratorTarget("cuda", "sm100").supports_tcgen05_int8
    assert AcceleratorTarget("CUDA", "SM100:a").supports_tcgen05_int8
    for arch in ("sm90", "sm120", "sm89", "sm103", None):
        assert not AcceleratorTarget("cuda", arch).supports_tcgen05_int8
    assert not AcceleratorTarget("cpu").supports_tcgen05_int8
    assert AcceleratorTarget.from_device(torch.device("cpu")).backend == "cpu"


@pytest.mark.parametrize("dtype", [torch.float32, torch.int8])
def test_rejects_unsupported_dtype(dtype: torch.dtype) -> None:
    q = torch.zeros((1, 1, 8, 64), dtype=dtype)
    with pytest.raises(ValueError, match="float16 or bfloat16"):
        piper_attention(q, q, q)


def test_rejects_mismatched_dtypes() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="share a dtype"):
        piper_attention(q, k.to(torch.bfloat16), v)


def test_rejects_unsupported_head_dimension() -> None:
    q = torch.randn(1, 1, 8, 32, dtype=torch.float16)
    with pytest.raises(ValueError, match="head dimensions 64 and 128"):
        piper_attention(q, q, q)


def test_rejects_mismatched_key_value_lengths() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="key/value lengths"):
        piper_attention(q, k, v[:, :, :-1])


def test_rejects_rectangular_causal_inputs() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="equal query and key lengths"):
        piper_attention(q[:, :, :-1], k, v, is_causal=True)


@pytest.mark.parametrize(("nq", "nk"), [(0, 8), (8, 0)])
def test_rejects_empty_sequences(nq: int, nk: int) -> None:
    q = torch.empty((1, 1, nq, 64), dtype=torch.float16)
    k = torch.empty((1, 1, nk, 64), dtype=torch.float16)
    with pytest.raises(ValueError, match="does not accept empty"):
        piper_attention(q, k, k)


def test_rejects_noncontiguous_head_dimension() -> None:
    storage = torch.randn(1, 1, 8, 128, dtype=torch.float16)
    q = storage[..., ::2]
    with pytest.raises(ValueError, match="head dimension must be contiguous"):
        piper_attention(q, q, q)


def test_rejects_autograd() -> None:
    q, k, v = _inputs()
    q.requires_grad_(True)
    with pytest.raises(RuntimeError, match="inference-only"):
        piper_attention(q, k, v)


@pytest.mark.parametrize("scale", [0.0, -1.0, float("inf"), float("nan")])
def test_rejects_invalid_scale(scale: float) -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match="finite and positive"):
        piper_attention(q, k, v, scale=scale)


def test_rejects_wrong_rank_and_mismatched_heads() -> None:
    q, k, v = _inputs()
    with pytest.raises(ValueError, match=r"must have shape \[batch, heads, sequence, head_dim\]"):
        piper_attention(q[0], k, v)
    with pytest.raises(ValueError, match="equal batch and head dimensions"):
        piper_attention(q, k[:, :1], v[:, :1])
