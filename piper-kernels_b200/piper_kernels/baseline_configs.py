"""Seeded synthetic inputs for the five headline Piper Attention workloads.

The reference measures on synthetic seeded tensors too (Piper Kernels 0.2.1,
``benchmarks/lib/attention.py:99-121``); no dataset is involved.  Each
workload fixes a shape, a dtype, the causal flag and the value distribution:

==========  ===========================  =====  ======  ===============================================
name        B, H, N, D                   dtype  causal  distribution
==========  ===========================  =====  ======  ===============================================
c1          1, 2, 256, 64                fp16   no      Q,K,V ~ N(0,1); K += c[d], c ~ N(0, 3^2)
c2          2, 24, 4096, 128             bf16   no      Q,K ~ N(0,1), 4 K channels +8; V += b[d], b ~ N(0, 2^2)
c3          4, 32, 8192, 128             fp16   yes     Q,K,V ~ N(0,1); K += c[d], c ~ N(0, 2^2)
c4          1, 40, 16384, 128            bf16   no      Q,K,V ~ N(0,1); V += b[d], b ~ N(0,1)
c5          1, 24, 131072, 128           bf16   no      Q,K,V ~ N(0,1); V += b[d], b ~ N(0,1)  (ring)
c5causal    1, 24, 131072, 128           bf16   yes     as c5, causal (zig-zag ring; not a headline config)
==========  ===========================  =====  ======  ===============================================

Offsets are per-(b, h) channel vectors shared over the tokens.  Every rank of
a multi-GPU run generates the same global problem from the same seed (the
CUDA generator is deterministic across devices) and takes its part of it, so
the union of the ranks' work is bit-identical to the one-GPU problem.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

DEFAULT_SEED = 1000


@dataclass(frozen=True)
class BaselineConfig:
    name: str
    batch: int
    heads: int
    seq_len: int
    head_dim: int
    dtype: torch.dtype
    is_causal: bool
    description: str

    @property
    def shape(self) -> tuple[int, int, int, int]:
        return (self.batch, self.heads, self.seq_len, self.head_dim)


CONFIGS: dict[str, BaselineConfig] = {
    c.name: c
    for c in (
        BaselineConfig("c1", 1, 2, 256, 64, torch.float16, False,
                       "piper_attention non-causal B1 H2 N256 D64 fp16 (BASELINE configs[0]); K offset ~N(0,3^2)"),
        BaselineConfig("c2", 2, 24, 4096, 128, torch.bfloat16, False,
                       "piper_attention non-causal B2 H24 N4096 D128 bf16 (BASELINE configs[1]); "
                       "4 K outlier channels +8, V bias ~N(0,2^2)"),
        BaselineConfig("c3", 4, 32, 8192, 128, torch.float16, True,
                       "piper_attention causal B4 H32 N8192 D128 fp16 (BASELINE configs[2]); K offset ~N(0,2^2)"),
        BaselineConfig("c4", 1, 40, 16384, 128, torch.bfloat16, False,
                       "piper_attention non-causal B1 H40 N16384 D128 bf16 (BASELINE configs[3]); V bias ~N(0,1)"),
        BaselineConfig("c5", 1, 24, 131072, 128, torch.bfloat16, False,
                       "piper_attention non-causal sequence-sharded ring B1 H24 N131072 D128 bf16 "
                       "(BASELINE configs[4]); V bias ~N(0,1)"),
        BaselineConfig("c5causal", 1, 24, 131072, 128, torch.bfloat16, True,
                       "piper_attention CAUSAL sequence-sharded ring, zig-zag shards, B1 H24 N131072 D128 bf16 "
                       "(the c5 shape with the causal mask; not a BASELINE config)"),
    )
}


def make_inputs(name: str, device: torch.device | str, *,
                seed: int = DEFAULT_SEED) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The seeded global ``[B, H, N, D]`` query, key and value of workload ``name``.

    Values are drawn in fp32 from ``torch.Generator(device)`` in a fixed order
    (Q, K, V, then the offsets) and rounded once to the workload's dtype.
    """
    cfg = CONFIGS[name]
    device = torch.device(device)
    g = torch.Generator(device=device).manual_seed(seed)
    b, h, n, d = cfg.shape
    shape = (b, h, n, d)

    def randn(*size: int) -> torch.Tensor:
        return torch.randn(size, generator=g, device=device, dtype=torch.float32)

    q = randn(*shape).to(cfg.dtype)
    k = randn(*shape)
    v = randn(*shape)
    if name == "c1":
        k += randn(b, h, 1, d) * 3.0
    elif name == "c2":
        channels = torch.randperm(d, generator=g, device=device)[:4]
        k[..., channels] += 8.0
        v += randn(b, h, 1, d) * 2.0
    elif name == "c3":
        k += randn(b, h, 1, d) * 2.0
    else:  # c4, c5, c5causal
        v += randn(b, h, 1, d)
    return q, k.to(cfg.dtype), v.to(cfg.dtype)
