"""Attention plugin package: registry, the ``sqrt_block`` plugin and a GPT-2 caller."""

from .attention_registry import (BaseAttention, available_attentions, build_attention,
                                 get_attention, register_attention)

__all__ = ["BaseAttention", "available_attentions", "build_attention", "get_attention",
           "register_attention"]
