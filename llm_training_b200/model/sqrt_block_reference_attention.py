"""The reference's own sqrt-block attention semantics, as a CUDA-backed plugin.

Registered as ``sqrt_block_reference``.  Same constructor, parameters
(``Wq, Wk, Wv, c_proj``) and ``forward(X: (B, T, C)) -> (B, T, C)`` as the
reference's ``CustomAttention`` (model/custom_attention.py:138-230), and the
same attention core: a causal softmax map inside each block, one summary per
block (the column sums of its map), a softmax over strictly earlier blocks'
summaries and the own block added at weight 1 (:183-227, _ScaledBlockCombine
:82-135).  The core runs in ``sqb_refsem_fwd`` / ``sqb_refsem_bwd``; T must be a
perfect square (``block_geometry``, :68-79), as in the reference.

This is the mode to use where a model trained with the reference's module is to
be run or fine-tuned unchanged.  The ``sqrt_block`` plugin implements the
two-level operator with mean-pooled summaries in one softmax instead.
"""

from __future__ import annotations

import torch.nn as nn

from ..ops import reference_attention
from .attention_registry import BaseAttention, register_attention


@register_attention("sqrt_block_reference")
class ReferenceSqrtBlockAttention(BaseAttention):
    """The reference's sqrt_block math on the CUDA library; same in, same out."""

    def __init__(self, config):
        super().__init__(config)
        assert config.n_embd % config.n_head == 0
        self.Wq = nn.Linear(config.n_embd, config.n_embd, bias=config.bias)
        self.Wk = nn.Linear(config.n_embd, config.n_embd, bias=config.bias)
        self.Wv = nn.Linear(config.n_embd, config.n_embd, bias=config.bias)
        self.c_proj = nn.Linear(config.n_embd, config.n_embd, bias=config.bias)
        self.attn_dropout = nn.Dropout(config.dropout)
        self.resid_dropout = nn.Dropout(config.dropout)
        self.n_head = config.n_head
        self.block_size = config.block_size
        self.attn_pdrop = float(config.dropout or 0.0)

    def forward(self, X):
        Batch, Token, Embedding = X.shape
        assert Token <= self.block_size, (
            f"sequence length {Token} exceeds block_size {self.block_size}")
        if self.training and self.attn_pdrop > 0:
            raise NotImplementedError(
                "sqrt_block_reference attention does not implement attention-map dropout; "
                "use dropout=0.0")
        head_dim = Embedding // self.n_head
        shape = (Batch, Token, self.n_head, head_dim)
        q = self.Wq(X).view(shape)
        k = self.Wk(X).view(shape)
        v = self.Wv(X).view(shape)
        y = reference_attention(q, k, v)
        y = self.c_proj(y.reshape(Batch, Token, Embedding))
        return self.resid_dropout(y)
