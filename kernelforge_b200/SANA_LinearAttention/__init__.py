"""SANA ReLU linear attention (drop-in for SANA_LinearAttention/__init__.py:3-12)."""

from .custom import QKVAttnMatmul, qkv_attn_matmul, sana_linattn_into

__all__ = ["QKVAttnMatmul", "qkv_attn_matmul", "sana_linattn_into"]
