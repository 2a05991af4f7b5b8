"""SageAttention2++ (8+8): public operator and its B200 backend."""

from .dispatch import sage_attention_2pp

__all__ = ["sage_attention_2pp"]
