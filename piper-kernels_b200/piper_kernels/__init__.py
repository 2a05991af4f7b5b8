"""Piper Kernels -- B200 (sm_100a) backend of the Piper Attention operator.

Drop-in for the reference package's public attention entry point
(Piper Kernels 0.2.1, ``src/piper_kernels/__init__.py:3-6``): the same
``piper_kernels.piper_attention`` function and the same
``torch.ops.piper_kernels.piper_attention`` custom operator, computed by
hand-written sm_100a CUDA kernels behind the C ABI in ``include/piper_b200.h``.
"""

from .attention.piper_attention import piper_attention

__all__ = ["piper_attention"]
