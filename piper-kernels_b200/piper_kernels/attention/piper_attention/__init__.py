"""Piper Attention: public operator and its B200 backend."""

from .dispatch import piper_attention
from .ring import ring_piper_attention

__all__ = ["piper_attention", "ring_piper_attention"]
