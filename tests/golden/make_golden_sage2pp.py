"""Generate the SageAttention2++ golden fixtures by running the reference itself.

Usage (in a container that has the reference source tree; the .npz files are
committed and the reference is not needed afterwards)::

    python tests/golden/make_golden_sage2pp.py --reference-src <path to piper-kernels/src>

For each case it stores the fp16/bf16 inputs (raw 16-bit patterns) and what
the reference's portable implementation returns for them:

* ``reference_sage_attention_2pp(q, k, v, scale, is_causal)`` with the default
  ``qk_quantization="per_thread"`` (src/piper_kernels/attention/
  sage_attention_2pp/reference.py:30-104), the output;
* ``quantize_query_key(q, k, granularity="per_thread")``
  (qk_quantization/int8/sage/reference.py:23-60, 80-108): Q/K codes and their
  per-row / per-key scales;
* ``_quantize_value_per_channel(v)`` (sage_attention_2pp/reference.py:21-24):
  the FP8 e4m3 V bytes and the per-channel scales;
* the K sequence mean as the reference computes it (fp32 ``mean``), which
  the Q/K codes depend on.

Inputs are seeded synthetic tensors shaped like the reference's own tests
(tests/attention/sage_attention_2pp/test_reference.py, test_triton.py).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CASES = {
    # name: (B, H, Nq, Nk, D, dtype, causal, seed, key offset, value offset)
    "s2pp_n193_d128_bf16_noncausal": (1, 2, 193, 193, 128, torch.bfloat16, False, 43, 0.0, 0.0),
    "s2pp_n193_d128_bf16_causal": (1, 2, 193, 193, 128, torch.bfloat16, True, 44, 0.0, 0.0),
    "s2pp_n193_d64_fp16_noncausal": (1, 2, 193, 193, 64, torch.float16, False, 45, 0.0, 0.0),
    "s2pp_n65_d64_fp16_causal": (1, 2, 65, 65, 64, torch.float16, True, 41, 0.0, 0.0),
    "s2pp_rect_q17_k29_d64_bf16": (2, 1, 17, 29, 64, torch.bfloat16, False, 42, 0.0, 0.0),
    "s2pp_offsets_n320_d128_bf16": (1, 2, 320, 320, 128, torch.bfloat16, False, 46, 2.0, 1.0),
}


def case_inputs(name: str):
    b, h, nq, nk, d, dt, causal, seed, koff, voff = CASES[name]
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((b, h, nq, d), generator=g)
    k = torch.randn((b, h, nk, d), generator=g) + torch.randn((b, h, 1, d), generator=g) * koff
    v = torch.randn((b, h, nk, d), generator=g) + torch.randn((b, h, 1, d), generator=g) * voff
    return q.to(dt), k.to(dt), v.to(dt), causal


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", required=True)
    args = parser.parse_args()
    sys.path.insert(0, args.reference_src)
    from piper_kernels.attention.kernels.qk_quantization.int8.sage.reference import quantize_query_key
    from piper_kernels.attention.sage_attention_2pp.reference import (
        _quantize_value_per_channel,
        reference_sage_attention_2pp,
    )

    for name in CASES:
        q, k, v, causal = case_inputs(name)
        scale = q.shape[-1] ** -0.5
        out = reference_sage_attention_2pp(q, k, v, scale, causal)
        q8, k8, qs, ks = quantize_query_key(q, k, granularity="per_thread")
        v8, vs = _quantize_value_per_channel(v)
        np.savez_compressed(
            HERE / f"{name}.npz",
            query=q.view(torch.int16).numpy(), key=k.view(torch.int16).numpy(), value=v.view(torch.int16).numpy(),
            dtype=np.array(str(q.dtype).replace("torch.", "")), is_causal=np.array(causal), scale=np.array(scale),
            out=out.float().numpy(), query_int8=q8.numpy(), key_int8=k8.numpy(),
            query_scale=qs.float().numpy(), key_scale=ks.float().numpy(),
            value_fp8=v8.view(torch.uint8).numpy(), value_scale=vs.float().numpy(),
            key_mean=k.float().mean(dim=2).numpy(),
        )
        print(name, out.shape)


if __name__ == "__main__":
    main()
