"""The ``sqrt_block`` attention plugin backed by the sm_100a CUDA library.

Drop-in for the reference's registered ``sqrt_block`` / ``custom`` module
(model/custom_attention.py:138-230): same constructor (reads n_embd, n_head,
block_size, bias, dropout from the config, :142-153), same parameters
``Wq, Wk, Wv, c_proj`` (:145-149) so state dicts and checkpoints carry over,
no persistent buffers (:161-173 registers its masks persistent=False), and the
same ``forward(X: (B, T, C)) -> (B, T, C)``.

What changes is the attention core between the projections and c_proj
(:183-227).  Here it is the two-level operator: each query attends causally to
its own block of b tokens and to the mean-pooled K/V of every earlier complete
block, in one softmax, computed by ``sqb_fwd`` / ``sqb_bwd``.  On CUDA the three
projections run as one GEMM over Wq/Wk/Wv stacked, and the thirds of its (B, T, 3C)
output are handed to the kernels as strided (B, T, H, D) views, so the reference's
permute copies (:188-191, :227) disappear, and the backward writes dQ, dK, dV into
one packed gradient (one GEMM for dX, no gradient adds).

The block length is ``config.sqrt_block_b`` when set, else
b = round_up(ceil(sqrt(T)), 16) of the running sequence length; unlike the
reference's block_geometry (:68-79) any T >= 1 is accepted.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import sqrt_block_attention, sqrt_block_attention_qkv
from .attention_registry import BaseAttention, register_attention


@register_attention("sqrt_block", "custom")
class SqrtBlockAttention(BaseAttention):
    """Two-level sqrt-block causal attention; same in, same out as the reference module."""

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
        self.block = getattr(config, "sqrt_block_b", None)
        self.impl = getattr(config, "sqrt_block_impl", "auto")
        # Attention-probability dropout is not part of the fused operator; the
        # reference trains with dropout 0.0 (GPT_Config.py:11).  Output dropout
        # (resid_dropout) still applies.
        self.attn_pdrop = float(config.dropout or 0.0)

    def forward(self, X):
        Batch, Token, Embedding = X.shape
        assert Token <= self.block_size, (
            f"sequence length {Token} exceeds block_size {self.block_size}")
        if self.training and self.attn_pdrop > 0:
            raise NotImplementedError(
                "sqrt_block attention does not implement attention-probability dropout; "
                "use dropout=0.0")
        head_dim = Embedding // self.n_head
        if X.is_cuda:
            # Q, K and V from one GEMM over the three weights stacked (the same
            # dot products as Wq/Wk/Wv applied one by one): the kernels read the
            # packed (B, T, 3C) output in place and the backward hands back one
            # packed gradient, so dX is one GEMM with no gradient adds
            weight = torch.cat((self.Wq.weight, self.Wk.weight, self.Wv.weight))
            bias = (torch.cat((self.Wq.bias, self.Wk.bias, self.Wv.bias))
                    if self.Wq.bias is not None else None)
            qkv = F.linear(X, weight, bias)
            y = sqrt_block_attention_qkv(qkv, self.n_head, self.block, None, self.impl)
        else:
            shape = (Batch, Token, self.n_head, head_dim)
            q = self.Wq(X).view(shape)
            k = self.Wk(X).view(shape)
            v = self.Wv(X).view(shape)
            y = sqrt_block_attention(q, k, v, self.block, None, self.impl)
        y = self.c_proj(y.view(Batch, Token, Embedding))
        return self.resid_dropout(y)
