"""Model configuration, field-compatible with the reference's GPT_Config.ModelConfig
(GPT_Config.py:4-17) plus the sqrt-block block length.

``sqrt_block_b``: block length b of the sqrt-block attention; None selects
b = round_up(ceil(sqrt(T)), 16) for the running sequence length T.
``sqrt_block_impl``: kernel family, "auto" (tcgen05 where supported), "simt"
or "tcgen05".
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


@dataclass
class ModelConfig:
    block_size: int = 1024
    vocab_size: int = 50304
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    dropout: float = 0.0
    bias: bool = True
    attention: str = "sqrt_block"
    sqrt_block_b: Optional[int] = None
    sqrt_block_impl: str = "auto"


def gpt2_small(**kw) -> ModelConfig:
    """GPT-2 small as trained with sqrt-block attention: 12L/12H/768, bias-free
    LayerNorms and Linears, vocab 50257, context 1024."""
    base = dict(block_size=1024, vocab_size=50257, n_layer=12, n_head=12, n_embd=768,
                bias=False, attention="sqrt_block")
    base.update(kw)
    return ModelConfig(**base)


def gpt2_medium(**kw) -> ModelConfig:
    """GPT-2 medium: 24L/16H/1024, bias-free, vocab 50257; context set by the caller."""
    base = dict(block_size=8192, vocab_size=50257, n_layer=24, n_head=16, n_embd=1024,
                bias=False, attention="sqrt_block")
    base.update(kw)
    return ModelConfig(**base)
