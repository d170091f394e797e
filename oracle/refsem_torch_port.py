"""PyTorch CPU restatement of the reference's own sqrt-block attention core.
TEST INFRASTRUCTURE ONLY: the timed reference arm of ``bench.py --workload
refsem-cfg2`` (never imported by the product path).

The reference's registered ``sqrt_block`` module (model/custom_attention.py:138)
is itself a sequence of PyTorch tensor ops; its file cannot travel to the GPU
box where the benchmark runs, so the same core is restated here with the same
ops on the same blocked layout, and autograd for the backward:

* blocked view (B, H, G, L, d), G = L = sqrt(T)   (custom_attention.py:188-191)
* local = causal softmax of Q K^T / sqrt(d)         (:195-198)
* summary = local.sum(-2)                            (:203)
* glob = softmax(strict-mask(summary summary^T / sqrt(L))), NaN -> 0   (:209-213)
* out = P + glob P with P = local V                  (_ScaledBlockCombine, :106-109)

``oracle/refsem_oracle.py`` (float64 numpy, pinned to fixtures made by running
the reference module) checks this port in the CPU tests.
"""

from __future__ import annotations

import math

import torch


def reference_core(q, k, v, scale=None):
    """q, k, v: (B, H, T, D) CPU tensors, T a perfect square -> out (B, H, T, D)."""
    B, H, T, D = q.shape
    L = math.isqrt(T)
    if L * L != T:
        raise ValueError(f"sequence length {T} must be a perfect square")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    G = L
    qb, kb, vb = (x.reshape(B, H, G, L, D) for x in (q, k, v))
    scores = torch.matmul(qb, kb.transpose(-2, -1)) * scale
    causal = torch.ones(L, L, dtype=torch.bool).tril()
    local = torch.softmax(scores.masked_fill(~causal, float("-inf")), dim=-1)
    summary = local.sum(dim=-2)                                   # (B, H, G, L)
    gs = torch.matmul(summary, summary.transpose(-2, -1)) / math.sqrt(L)
    strict = torch.ones(G, G, dtype=torch.bool).tril(-1)
    glob = torch.nan_to_num(torch.softmax(gs.masked_fill(~strict, float("-inf")), dim=-1))
    p = torch.matmul(local, vb)                                   # (B, H, G, L, D)
    out = p + torch.einsum("bhij,bhjld->bhild", glob, p)
    return out.reshape(B, H, T, D)
