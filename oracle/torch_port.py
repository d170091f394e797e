"""Batched PyTorch CPU restatement of sqrt-block attention.  TEST INFRASTRUCTURE ONLY.

Used as (a) the fp32/fp64 autograd reference in the tests and (b) the timed CPU
baseline of ``bench.py`` (``cpu_baseline`` and ``--impl reference``).  It is the
"port" kind of baseline: the reference repository has no CPU implementation of
this operator (its ``sqrt_block``, model/custom_attention.py:175-230, computes
column-sum summaries with a G x G softmax instead), so the operator is restated
here with the same tensor-op style the reference uses there - batched
``torch.matmul`` over a blocked (B, H, G, b, D) view (custom_attention.py:188-198)
- and autograd for the backward.  Never imported by the product path.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .sqrtblock_oracle import geometry


def sqrt_block_attention_ref(q, k, v, b=None, scale=None):
    """q, k, v: (B, H, T, D) CPU tensors -> (o, lse).  Differentiable."""
    B, H, T, D = q.shape
    b, G, Gc = geometry(T, b)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    pad = G * b - T
    if pad:
        q = F.pad(q, (0, 0, 0, pad))
        k = F.pad(k, (0, 0, 0, pad))
        v = F.pad(v, (0, 0, 0, pad))
    qb = q.view(B, H, G, b, D)
    kb = k.view(B, H, G, b, D)
    vb = v.view(B, H, G, b, D)
    kbar = kb[:, :, :Gc].mean(dim=-2)  # (B, H, Gc, D)
    vbar = vb[:, :, :Gc].mean(dim=-2)
    s_in = torch.matmul(qb, kb.transpose(-2, -1)) * scale  # (B, H, G, b, b)
    causal = torch.ones(b, b, dtype=torch.bool).tril()
    s_in = s_in.masked_fill(~causal, float("-inf"))
    s_x = torch.matmul(qb, kbar.unsqueeze(2).transpose(-2, -1)) * scale  # (B,H,G,b,Gc)
    blk = torch.arange(G).view(G, 1, 1)
    j = torch.arange(Gc).view(1, 1, Gc)
    s_x = s_x.masked_fill(~(j < blk), float("-inf"))
    s = torch.cat([s_in, s_x], dim=-1)
    lse = torch.logsumexp(s, dim=-1)  # (B, H, G, b)
    p = torch.exp(s - lse.unsqueeze(-1))
    o = torch.matmul(p[..., :b], vb) + torch.matmul(p[..., b:], vbar.unsqueeze(2))
    o = o.reshape(B, H, G * b, D)[:, :, :T]
    lse = lse.reshape(B, H, G * b)[:, :, :T]
    return o, lse
