"""Attention operators (B200 backend)."""
