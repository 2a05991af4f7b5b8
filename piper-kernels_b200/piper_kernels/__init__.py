"""Piper Kernels -- B200 (sm_100a) backend of the attention operators.

Drop-in for the reference package's public entry points
(Piper Kernels 0.2.1, ``src/piper_kernels/__init__.py:3-6``): the same
``piper_kernels.piper_attention`` and ``piper_kernels.sage_attention_2pp``
functions and the same ``torch.ops.piper_kernels.*`` custom operators,
computed by hand-written sm_100a CUDA kernels behind the C ABI in
``include/piper_b200.h``.
"""

from .attention.piper_attention import piper_attention
from .attention.sage_attention_2pp import sage_attention_2pp

__all__ = ["piper_attention", "sage_attention_2pp"]
