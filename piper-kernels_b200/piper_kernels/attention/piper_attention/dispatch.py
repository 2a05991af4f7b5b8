"""Public Piper Attention operator: validation, then the B200 backend.

Same signature and validation as the reference
(Piper Kernels 0.2.1, ``src/piper_kernels/attention/piper_attention/dispatch.py:39-83``).
One deliberate difference: the reference falls back to its slow portable
PyTorch implementation on devices its Triton backend does not support
(dispatch.py:77-83).  This package is the B200 backend only and has no CPU or
generic-GPU fallback, so such calls raise ``RuntimeError`` instead of silently
running elsewhere.
"""

from __future__ import annotations

import torch

from ..._targets import AcceleratorTarget
from .._validation import validate_attention_inputs
from .b200 import b200_piper_attention

OPERATOR = "Piper Attention"


def piper_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
    is_causal: bool = False,
) -> torch.Tensor:
    """Run Piper Attention's key-scaled UINT8-P/INT8-V forward attention.

    Query, key and value use ``[batch, heads, sequence, head_dim]`` layout with
    FP16 or BF16 elements and a contiguous head dimension (64 or 128).  Query
    and key lengths may differ for non-causal attention.  ``scale`` defaults to
    ``head_dim ** -0.5``.

    K is smoothed by its sequence mean; Q and K are quantized to INT8 with one
    scale per 32 query rows / 64 key rows; QK^T runs as INT8 tensor-core MMAs
    with an FP32 online softmax over 64-key blocks; each V key row gets its own
    signed-INT8 scale, folded into nonnegative UINT8 probability codes for a
    UINT8xINT8 PV MMA.  Non-causal calls centre V by its sequence mean and add
    it back in the epilogue; causal calls leave V uncentered.  Inference only.
    """
    converted_scale = validate_attention_inputs(OPERATOR, query, key, value, scale, is_causal)
    target = AcceleratorTarget.from_device(query.device)
    if not target.supports_tcgen05_int8:
        raise RuntimeError(
            f"{OPERATOR}'s B200 backend requires CUDA tensors on an sm_100 GPU, "
            f"got device {query.device} ({target.architecture or target.backend}); "
            "this package has no CPU or generic-GPU fallback"
        )
    return b200_piper_attention(query, key, value, converted_scale, is_causal)
