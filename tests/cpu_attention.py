"""A dense causal attention plugin that runs on CPU, for host-side trainer tests only
(the sqrt-block op itself has no CPU path)."""

import torch.nn as nn
import torch.nn.functional as F

from llm_training_b200.model.attention_registry import BaseAttention


class CausalAttentionCPU(BaseAttention):
    def __init__(self, config):
        super().__init__(config)
        C = config.n_embd
        self.Wq = nn.Linear(C, C, bias=config.bias)
        self.Wk = nn.Linear(C, C, bias=config.bias)
        self.Wv = nn.Linear(C, C, bias=config.bias)
        self.c_proj = nn.Linear(C, C, bias=config.bias)
        self.n_head = config.n_head

    def forward(self, X):
        B, T, C = X.shape
        sh = (B, T, self.n_head, C // self.n_head)
        q, k, v = [f(X).view(sh).transpose(1, 2) for f in (self.Wq, self.Wk, self.Wv)]
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.c_proj(y.transpose(1, 2).reshape(B, T, C))
