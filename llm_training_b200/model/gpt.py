"""Minimal GPT-2 caller of the attention plugin (training configurations only).

Mirrors the reference's model stack so that state-dict keys and numerics of the
non-attention parts match: ``GPT`` (model/GPT.py:11-70: wte/wpe/drop/attn_blocks/
ln_ in ``transformer``, tied ``lm_head``, N(0, 0.02) init, c_proj scaled by
1/sqrt(2 n_layer)), ``Attention_Block`` (model/attention_block.py:6-25, pre-norm
``x + attn(lm1(x)); x + mlp(lm2(x))``), ``MLP`` (model/mlp.py:5-16, tanh GELU)
and ``LayerNorm`` (model/layer_norm.py:4-13, optional bias).  The attention is
built through ``build_attention(config)`` exactly as the reference block does.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import add_layer_norm, add_layer_norm_supported, layer_norm, layer_norm_supported
from .attention_registry import build_attention


class LayerNorm(nn.Module):
    def __init__(self, ndim, bias=True, eps=1e-5):
        super().__init__()
        self.ln = nn.LayerNorm(ndim, eps=eps)
        if not bias:
            self.ln.register_parameter("bias", None)

    @staticmethod
    def _out_dtype():
        out = torch.float32
        if torch.is_autocast_enabled("cuda"):
            out = torch.get_autocast_dtype("cuda")
        return out if out in (torch.float32, torch.bfloat16) else None

    def forward(self, x):
        # CUDA fp32 rows (the residual stream): the library's fused LayerNorm,
        # fp32 math as nn.LayerNorm under autocast, its output written directly
        # in the autocast dtype that every consumer here (a Linear) casts it to
        if layer_norm_supported(x, self.ln.weight):
            out = self._out_dtype()
            if out is not None:
                return layer_norm(x, self.ln.weight, self.ln.bias, self.ln.eps, out)
        return self.ln(x)

    def add_forward(self, x, h):
        """(x + h, this LayerNorm of x + h): the residual add and the LayerNorm
        that reads its sum, as one kernel each way on the CUDA fp32 residual
        stream (the same fp32 sum and LayerNorm as the two separate ops)."""
        if add_layer_norm_supported(x, h, self.ln.weight):
            out = self._out_dtype()
            if out is not None:
                return add_layer_norm(x, h, self.ln.weight, self.ln.bias, self.ln.eps, out)
        x = x + h
        return x, self(x)


class MLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.c_fc = nn.Linear(config.n_embd, 4 * config.n_embd, bias=config.bias)
        self.gelu = nn.GELU(approximate="tanh")
        self.c_proj = nn.Linear(4 * config.n_embd, config.n_embd, bias=config.bias)
        self.drop = nn.Dropout(config.dropout)

    def forward(self, x):
        return self.drop(self.c_proj(self.gelu(self.c_fc(x))))


class Attention_Block(nn.Module):  # noqa: N801  (reference class name)
    def __init__(self, config):
        super().__init__()
        self.lm1 = LayerNorm(config.n_embd, bias=config.bias)
        self.attn = build_attention(config)
        self.lm2 = LayerNorm(config.n_embd, bias=config.bias)
        self.mlp = MLP(config)

    def forward(self, x):
        x = x + self.attn(self.lm1(x))
        x = x + self.mlp(self.lm2(x))
        return x


class GPT(nn.Module):
    def __init__(self, config):
        super().__init__()
        assert config.vocab_size is not None
        assert config.block_size is not None
        self.config = config
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(config.vocab_size, config.n_embd),
            wpe=nn.Embedding(config.block_size, config.n_embd),
            drop=nn.Dropout(config.dropout),
            attn_blocks=nn.ModuleList([Attention_Block(config) for _ in range(config.n_layer)]),
            ln_=LayerNorm(config.n_embd, bias=config.bias),
        ))
        self.lm_head = nn.Linear(config.n_embd, config.vocab_size, bias=False)
        self.transformer.wte.weight = self.lm_head.weight
        self.apply(self._init_weights)
        for pn, p in self.named_parameters():
            if pn.endswith("c_proj.weight"):
                torch.nn.init.normal_(p, mean=0.0, std=0.02 / math.sqrt(2 * config.n_layer))

    @staticmethod
    def _init_weights(module):
        if isinstance(module, nn.Linear):
            torch.nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                torch.nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            torch.nn.init.normal_(module.weight, mean=0.0, std=0.02)

    # vocabulary rows are padded to this multiple in the logits GEMM (pad_vocab)
    VOCAB_ALIGN = 64

    def _vocab_pad_bias(self, device, dtype):
        """(Vp,): 0 for the real vocabulary, -inf for the padding (not a
        parameter and not in the state dict)."""
        V = self.config.vocab_size
        Vp = -(-V // self.VOCAB_ALIGN) * self.VOCAB_ALIGN
        bias = getattr(self, "_pad_bias", None)
        if bias is None or bias.device != device or bias.dtype != dtype or bias.numel() != Vp:
            bias = torch.zeros(Vp, device=device, dtype=dtype)
            bias[V:] = float("-inf")
            self.register_buffer("_pad_bias", bias, persistent=False)
        return bias

    def forward(self, idx, pad_vocab=False):
        """Logits (B, T, vocab).  With ``pad_vocab`` the logits are (B, T, Vp),
        Vp = vocab rounded up to a multiple of 64: the tied weight is zero-padded
        for the GEMM and the padded columns get -inf, so they take no probability
        and no gradient and a cross-entropy over them equals the unpadded one.
        The padding keeps every GEMM operand's leading dimension 16-byte aligned
        (vocab 50257 is odd, which sends these GEMMs to unaligned kernels several
        times slower); the parameters are unchanged."""
        b, t = idx.size()
        assert t <= self.config.block_size, (
            f"Cannot forward sequence of length {t}, block size is only {self.config.block_size}")
        pos = torch.arange(0, t, dtype=torch.long, device=idx.device)
        x = self.transformer.drop(self.transformer.wte(idx) + self.transformer.wpe(pos))
        # the blocks' residual stream (Attention_Block.forward, unrolled): each
        # residual add goes into the LayerNorm that next reads the stream - the
        # block's second one, the next block's first, or the final one
        blocks = self.transformer.attn_blocks
        h = (blocks[0].lm1 if len(blocks) else self.transformer.ln_)(x)
        for i, block in enumerate(blocks):
            x, y = block.lm2.add_forward(x, block.attn(h))
            nxt = blocks[i + 1].lm1 if i + 1 < len(blocks) else self.transformer.ln_
            x, h = nxt.add_forward(x, block.mlp(y))
        V = self.config.vocab_size
        if not pad_vocab or V % self.VOCAB_ALIGN == 0:
            return self.lm_head(h)
        bias = self._vocab_pad_bias(h.device, self.lm_head.weight.dtype)
        weight = F.pad(self.lm_head.weight, (0, 0, 0, bias.numel() - V))
        return F.linear(h, weight, bias)
