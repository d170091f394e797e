"""CPU oracle of the reference's own sqrt-block attention core.  TEST INFRASTRUCTURE ONLY.

Nothing in the product path imports this module: only the tests use it, as the
checker of the CUDA "reference semantics" mode (``sqb_refsem_fwd`` /
``sqb_refsem_bwd``).

This restates, in float64 numpy, the attention core of the module the reference
registers as ``sqrt_block`` / ``custom`` (model/custom_attention.py:138), per
batch n and head h, with T = G * L tokens and G = L = sqrt(T)
(``block_geometry``, custom_attention.py:68-79):

* local_i = softmax over keys m <= l of (Q_i K_i^T / sqrt(d))   (:195-198, causal,
  inclusive diagonal, one L x L map per block i);
* summary_i[m] = sum_l local_i[l, m]   (:203, column sums of the local map);
* glob[i, j] = softmax over j < i of (summary_i . summary_j / sqrt(L))   (:209-211,
  strictly earlier blocks), row 0 all zero (:212-213, NaN -> 0);
* P_i = local_i V_i and out_i = P_i + sum_{j<i} glob[i, j] P_j
  (_ScaledBlockCombine.forward, :99-109: the own block at weight 1, outside the
  softmax).

The backward is the analytic gradient of that composition: the combine's
hand-written backward (:111-135) for d_local, d_glob and dV, then the softmax
backward of glob and of local, with the summary's gradient reaching every row of
its block's local map.  Parity is pinned: tests/golden/make_golden.py runs the
reference module itself in float64 (its Q/K/V projections replaced by the seeded
leaf tensors, c_proj the identity) and stores its output and autograd gradients.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = ["geometry", "fwd", "bwd"]


def geometry(T: int):
    """(G, L) as custom_attention.py:68-79: T must be a perfect square."""
    L = math.isqrt(max(T, 0))
    if L * L != T or T <= 0:
        raise ValueError(f"sequence length {T} must be a perfect square")
    return L, L


def _local(q, k, scale):
    """(..., L, L) causal softmax maps of each block (custom_attention.py:195-198)."""
    L = q.shape[-2]
    s = np.einsum("...ld,...md->...lm", q, k) * scale
    s = np.where(np.tril(np.ones((L, L), dtype=bool)), s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    e = np.exp(s)
    return e / e.sum(-1, keepdims=True)


def _glob(summary, L):
    """(..., G, G) strictly-causal softmax among block summaries, row 0 zero
    (custom_attention.py:209-213)."""
    G = summary.shape[-2]
    gs = np.einsum("...im,...jm->...ij", summary, summary) / math.sqrt(L)
    mask = np.tril(np.ones((G, G), dtype=bool), k=-1)
    gs = np.where(mask, gs, -np.inf)
    mx = gs.max(-1, keepdims=True)
    mx = np.where(np.isfinite(mx), mx, 0.0)
    e = np.where(mask, np.exp(gs - mx), 0.0)
    den = e.sum(-1, keepdims=True)
    return np.where(den > 0, e / np.where(den > 0, den, 1.0), 0.0)


def _blocks(x, G, L):
    B, H, T, D = x.shape
    return x.reshape(B, H, G, L, D)


def fwd(q, k, v, scale=None):
    """q, k, v: (B, H, T, D) -> (out (B, H, T, D), glob (B, H, G, G), summary (B, H, G, L))."""
    q, k, v = (np.asarray(a, dtype=np.float64) for a in (q, k, v))
    B, H, T, D = q.shape
    G, L = geometry(T)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qb, kb, vb = (_blocks(a, G, L) for a in (q, k, v))
    local = _local(qb, kb, scale)                       # (B, H, G, L, L)
    summary = local.sum(-2)                             # (B, H, G, L)
    glob = _glob(summary, L)                            # (B, H, G, G)
    p = np.einsum("...lm,...md->...ld", local, vb)      # (B, H, G, L, D)
    out = p + np.einsum("...ij,...jld->...ild", glob, p)
    return out.reshape(B, H, T, D), glob, summary


def bwd(q, k, v, do, scale=None):
    """Gradients (dq, dk, dv), each (B, H, T, D), of sum(out * do)."""
    q, k, v, do = (np.asarray(a, dtype=np.float64) for a in (q, k, v, do))
    B, H, T, D = q.shape
    G, L = geometry(T)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qb, kb, vb, dob = (_blocks(a, G, L) for a in (q, k, v, do))
    local = _local(qb, kb, scale)
    summary = local.sum(-2)
    glob = _glob(summary, L)
    p = np.einsum("...lm,...md->...ld", local, vb)
    # combine (custom_attention.py:111-135): dP_j = dO_j + sum_i glob[i, j] dO_i,
    # d_glob[i, j] = <dO_i, P_j>
    dp = dob + np.einsum("...ij,...ild->...jld", glob, dob)
    dglob = np.einsum("...ild,...jld->...ij", dob, p)
    # glob softmax backward (masked entries and row 0 carry no gradient)
    dgs = glob * (dglob - (glob * dglob).sum(-1, keepdims=True))
    # gs[i, j] = s_i . s_j / sqrt(L): both factors are summaries
    dsum = (np.einsum("...ij,...jm->...im", dgs, summary) +
            np.einsum("...ji,...jm->...im", dgs, summary)) / math.sqrt(L)
    # local feeds P (through V) and the summary (every row of its block)
    dlocal = np.einsum("...ld,...md->...lm", dp, vb) + dsum[..., None, :]
    ds = local * (dlocal - (local * dlocal).sum(-1, keepdims=True))
    dq = np.einsum("...lm,...md->...ld", ds, kb) * scale
    dk = np.einsum("...lm,...ld->...md", ds, qb) * scale
    dv = np.einsum("...lm,...ld->...md", local, dp)
    return tuple(a.reshape(B, H, T, D) for a in (dq, dk, dv))
