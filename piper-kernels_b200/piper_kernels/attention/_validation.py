"""Input contract of the full-attention operators.

Mirrors the reference's checks and their user-facing messages
(Piper Kernels 0.2.1, ``src/piper_kernels/attention/_validation.py:1-102``) so
that callers see the same ``ValueError`` / ``RuntimeError`` text for the same
mistakes.  Everything here runs on the host before any device work.
"""

from __future__ import annotations

import math

import torch

SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)
SUPPORTED_HEAD_DIMS = (64, 128)


def _check_one(operator: str, name: str, tensor: torch.Tensor) -> None:
    # _validation.py:12-23
    if tensor.ndim != 4:
        raise ValueError(
            f"{operator} {name} must have shape [batch, heads, sequence, head_dim], "
            f"got {tuple(tensor.shape)}"
        )
    if tensor.dtype not in SUPPORTED_DTYPES:
        raise ValueError(f"{operator} {name} must use float16 or bfloat16, got {tensor.dtype}")
    if tensor.layout is not torch.strided:
        raise ValueError(f"{operator} {name} must use strided layout")
    if tensor.stride(-1) != 1:
        raise ValueError(f"{operator} {name}'s head dimension must be contiguous")


def _check_together(
    operator: str,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    is_causal: bool,
) -> None:
    # _validation.py:26-68
    devices = (query.device, key.device, value.device)
    if devices[0] != devices[1] or devices[0] != devices[2]:
        raise ValueError(
            f"{operator} query, key, and value must share a device, "
            f"got {devices[0]}/{devices[1]}/{devices[2]}"
        )
    if query.dtype is not key.dtype or query.dtype is not value.dtype:
        raise ValueError(
            f"{operator} query, key, and value must share a dtype, "
            f"got {query.dtype}/{key.dtype}/{value.dtype}"
        )
    if query.shape[:2] != key.shape[:2] or key.shape[:2] != value.shape[:2]:
        raise ValueError(
            f"{operator} currently requires equal batch and head dimensions, got "
            f"{query.shape[:2]}/{key.shape[:2]}/{value.shape[:2]}"
        )
    if key.shape[2] != value.shape[2]:
        raise ValueError(
            f"{operator} key/value lengths must match, got {key.shape[2]}/{value.shape[2]}"
        )
    if query.shape[3] != key.shape[3] or key.shape[3] != value.shape[3]:
        raise ValueError(
            f"{operator} head dimensions must match, got "
            f"{query.shape[3]}/{key.shape[3]}/{value.shape[3]}"
        )
    if query.shape[3] not in SUPPORTED_HEAD_DIMS:
        raise ValueError(
            f"{operator} currently supports head dimensions 64 and 128, got {query.shape[3]}"
        )
    if query.shape[2] == 0 or key.shape[2] == 0:
        raise ValueError(f"{operator} does not accept empty query or key sequences")
    if is_causal and query.shape[2] != key.shape[2]:
        raise ValueError(
            f"Causal {operator} currently requires equal query and key lengths, got "
            f"{query.shape[2]}/{key.shape[2]}"
        )


def validate_attention_inputs(
    operator: str,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scale: float | None,
    is_causal: bool,
) -> float:
    """Check the shared attention contract; return the effective softmax scale.

    The scale defaults to ``head_dim ** -0.5`` and must be finite and positive
    (``_validation.py:71-102``).
    """
    for name, tensor in (("query", query), ("key", key), ("value", value)):
        _check_one(operator, name, tensor)
    _check_together(operator, query, key, value, is_causal)
    if torch.is_grad_enabled() and (query.requires_grad or key.requires_grad or value.requires_grad):
        raise RuntimeError(f"{operator} is an inference-only operator and does not support autograd")
    effective = query.shape[-1] ** -0.5 if scale is None else float(scale)
    if not math.isfinite(effective) or effective <= 0:
        raise ValueError(f"{operator} scale must be finite and positive, got {scale}")
    return effective
