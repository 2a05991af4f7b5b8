"""Generate the golden fixtures by running the Piper Kernels reference itself.

Usage (in a container that has the reference source tree; it is not needed
afterwards -- the .npz files are committed)::

    python tests/golden/make_golden.py --reference-src <path to piper-kernels/src>

For every case it stores the fp16/bf16 inputs (raw 16-bit patterns), and what
the reference's portable implementation returns for them:

* ``reference_piper_attention(q, k, v, scale, is_causal, qk_quantization="per_warp")``
  (src/piper_kernels/attention/piper_attention/reference.py:35-118), the output;
* ``quantize_query_key(q, k, granularity="per_warp")``
  (src/piper_kernels/attention/kernels/qk_quantization/int8/sage/reference.py:80-108),
  the Q/K codes and per-group scales, plus the K sequence mean;
* ``_quantize_value_per_key`` (reference.py:22-32) on the centered V, the V codes
  and per-row scales, plus the V sequence mean (non-causal only).

Inputs are seeded synthetic tensors shaped like the reference's own tests
(tests/attention/piper_attention/test_reference.py, test_triton.py,
test_dispatch.py) and like the BASELINE configurations, scaled down.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _gen(seed: int):
    g = torch.Generator().manual_seed(seed)
    return g


def _randn(g, shape, scale=1.0):
    return torch.randn(shape, generator=g, dtype=torch.float32) * scale


def case_inputs(name: str):
    """Return (q, k, v, scale, is_causal) for a named case."""
    if name == "c1_b1h2n256d64_fp16":
        # K plus a per-channel offset ~N(0,3) shared over tokens.
        g = _gen(0)
        shape = (1, 2, 256, 64)
        q = _randn(g, shape)
        k = _randn(g, shape) + _randn(g, (1, 2, 1, 64), 3.0)
        v = _randn(g, shape)
        return q.half(), k.half(), v.half(), None, False
    if name.startswith("n193_"):
        # tests/attention/piper_attention/test_triton.py:111-145 (B1 H2 N193).
        d = 128 if "_d128_" in name else 64
        dt = torch.bfloat16 if "bf16" in name else torch.float16
        causal = name.endswith("_causal")
        g = _gen(54 + d + (1 if causal else 0))
        shape = (1, 2, 193, d)
        return _randn(g, shape).to(dt), _randn(g, shape).to(dt), _randn(g, shape).to(dt), None, causal
    if name == "rect_q9_k11_d64_fp16":
        # tests/attention/piper_attention/test_dispatch.py:23-34 (scale=0.2).
        g = _gen(50)
        q = _randn(g, (1, 1, 9, 64)).half()
        k = _randn(g, (1, 1, 11, 64)).half()
        v = _randn(g, (1, 1, 11, 64)).half()
        return q, k, v, 0.2, False
    if name == "const_v_n65_d64_fp16":
        # tests/attention/piper_attention/test_reference.py:42-57.
        g = _gen(52)
        q = _randn(g, (1, 2, 65, 64)).half()
        k = _randn(g, (1, 2, 65, 64)).half()
        v = _randn(g, (1, 2, 1, 64)).half().expand(1, 2, 65, 64).contiguous()
        return q, k, v, None, False
    if name == "large_v_n64_d64_fp16":
        # tests/attention/piper_attention/test_triton.py:245-266.
        q = torch.ones((1, 1, 64, 64), dtype=torch.float16)
        k = torch.ones_like(q)
        k[:, :, 0] = -1
        v = torch.ones_like(q)
        v[:, :, 0] = 40000
        return q, k, v, None, False
    if name == "c2like_b1h2n320d128_bf16":
        # BASELINE configs[1] distribution: 4 K outlier channels +8, V bias ~N(0,2).
        g = _gen(1)
        shape = (1, 2, 320, 128)
        q = _randn(g, shape)
        k = _randn(g, shape)
        channels = torch.randperm(128, generator=g)[:4]
        k[..., channels] += 8.0
        v = _randn(g, shape) + _randn(g, (1, 2, 1, 128), 2.0)
        return q.bfloat16(), k.bfloat16(), v.bfloat16(), None, False
    if name == "c3like_b1h2n256d128_fp16_causal":
        # BASELINE configs[2] distribution: K per-channel offset ~N(0,2), causal.
        g = _gen(2)
        shape = (1, 2, 256, 128)
        q = _randn(g, shape)
        k = _randn(g, shape) + _randn(g, (1, 2, 1, 128), 2.0)
        v = _randn(g, shape)
        return q.half(), k.half(), v.half(), None, True
    if name == "rect_q200_k333_d128_bf16":
        # Ragged, rectangular non-causal: neither length is a multiple of 32/64.
        g = _gen(3)
        q = _randn(g, (2, 1, 200, 128)).bfloat16()
        k = _randn(g, (2, 1, 333, 128)).bfloat16()
        v = (_randn(g, (2, 1, 333, 128)) + 0.5).bfloat16()
        return q, k, v, None, False
    raise KeyError(name)


CASES = [
    "c1_b1h2n256d64_fp16",
    "n193_d128_bf16_noncausal",
    "n193_d128_bf16_causal",
    "n193_d64_fp16_noncausal",
    "n193_d64_fp16_causal",
    "rect_q9_k11_d64_fp16",
    "const_v_n65_d64_fp16",
    "large_v_n64_d64_fp16",
    "c2like_b1h2n320d128_bf16",
    "c3like_b1h2n256d128_fp16_causal",
    "rect_q200_k333_d128_bf16",
]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", required=True)
    parser.add_argument("--out", default=str(HERE))
    args = parser.parse_args()
    sys.path.insert(0, args.reference_src)
    from piper_kernels.attention.kernels.qk_quantization.int8.sage.reference import (
        QUERY_BLOCK,
        KEY_BLOCK,
        quantize_per_group,
    )
    from piper_kernels.attention.piper_attention.reference import (
        _quantize_value_per_key,
        reference_piper_attention,
    )

    torch.set_num_threads(1)
    for name in CASES:
        q, k, v, scale, causal = case_inputs(name)
        eff_scale = q.shape[-1] ** -0.5 if scale is None else scale
        with torch.inference_mode():
            out = reference_piper_attention(q, k, v, eff_scale, causal, qk_quantization="per_warp")
            # The per-group scales before repeat_interleave (qk reference.py:90-102).
            kf = k.float()
            k_mean = kf.mean(dim=2, keepdim=True)
            q8, qs = quantize_per_group(q, QUERY_BLOCK, 127)
            k8, ks = quantize_per_group(kf - k_mean, KEY_BLOCK, 127)
            vf = v.float()
            v_mean = torch.zeros_like(vf[:, :, :1]) if causal else vf.mean(dim=2, keepdim=True)
            v8, vs = _quantize_value_per_key(vf - v_mean)
        dtype = "float16" if q.dtype is torch.float16 else "bfloat16"
        np.savez_compressed(
            Path(args.out) / f"{name}.npz",
            dtype=np.array(dtype),
            scale=np.array(eff_scale, np.float64),
            scale_given=np.array(scale is not None),
            is_causal=np.array(causal),
            query=_bits(q),
            key=_bits(k),
            value=_bits(v),
            out=_bits(out),
            query_int8=q8.numpy(),
            query_scale=qs.numpy(),
            key_int8=k8.numpy(),
            key_scale=ks.numpy(),
            key_mean=k_mean[:, :, 0].numpy(),
            value_int8=v8.numpy(),
            value_scale=vs.numpy(),
            value_mean=(v_mean[:, :, 0].numpy() if not causal else np.zeros(0, np.float32)),
        )
        print(name, tuple(q.shape), tuple(k.shape), dtype, "causal" if causal else "non-causal")


if __name__ == "__main__":
    main()
