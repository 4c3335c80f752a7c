"""FlashAttention forward / forward-mode JVP (drop-in for flash_attention_jvp/__init__.py:3-8)."""

from .custom import (
    FlashAttentionFunction,
    flash_attention,
    flash_attention_fwd_jvp,
    flash_attention_jvp,
    get_jvp_config,
)

__all__ = [
    "FlashAttentionFunction",
    "flash_attention",
    "flash_attention_fwd_jvp",
    "flash_attention_jvp",
    "get_jvp_config",
]
