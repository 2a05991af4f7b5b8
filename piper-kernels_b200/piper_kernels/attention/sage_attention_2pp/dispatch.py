"""Public SageAttention2++ operator: validation, then the B200 backend.

Same signature and validation as the reference
(Piper Kernels 0.2.1, ``src/piper_kernels/attention/sage_attention_2pp/dispatch.py:37-64``).
As for Piper Attention, the reference's portable PyTorch fallback on other
devices (dispatch.py:63-64) is not part of this package: such calls raise
``RuntimeError``.
"""

from __future__ import annotations

import torch

from ..._targets import AcceleratorTarget
from .._validation import validate_attention_inputs
from .b200 import b200_sage_attention_2pp

OPERATOR = "SageAttention2++"


def sage_attention_2pp(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
    is_causal: bool = False,
) -> torch.Tensor:
    """Run SageAttention2++ 8+8 forward attention.

    Query, key and value use ``[batch, heads, sequence, head_dim]`` layout with
    FP16 or BF16 elements and a contiguous head dimension (64 or 128).  Query
    and key lengths may differ for non-causal attention.  ``scale`` defaults to
    ``head_dim ** -0.5``.

    K is smoothed by its sequence mean; Q and K are quantized to INT8 with one
    scale per interleaved group of rows (4 of every 32 query rows, 16 of every
    64 key rows); QK^T runs as INT8 tensor-core MMAs with an FP32 online
    softmax over 64-key blocks; probabilities are stored as FP8 e4m3 against a
    running maximum shifted so the largest is 448; V is FP8 e4m3 with one scale
    per channel, and PV runs as an e4m3 x e4m3 tensor-core MMA with an FP32
    accumulator.  Inference only.
    """
    converted_scale = validate_attention_inputs(OPERATOR, query, key, value, scale, is_causal)
    target = AcceleratorTarget.from_device(query.device)
    if not target.supports_tcgen05_fp8:
        raise RuntimeError(
            f"{OPERATOR}'s B200 backend requires CUDA tensors on an sm_100 GPU, "
            f"got device {query.device} ({target.architecture or target.backend}); "
            "this package has no CPU or generic-GPU fallback"
        )
    return b200_sage_attention_2pp(query, key, value, converted_scale, is_causal)
