"""CPU checks of the reference-semantics oracle (oracle/refsem_oracle.py).

The oracle restates the reference's own sqrt_block attention core
(model/custom_attention.py:183-227, _ScaledBlockCombine :82-135).  It is pinned
to fixtures produced by running the reference module itself in float64
(tests/golden/make_golden.py: ``refsem_T256.npz``, ``refsem_T1024.npz``), and its
analytic backward is checked against central finite differences.
"""

import os

import numpy as np
import pytest

from oracle import refsem_oracle as rso

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def bhtd(a):
    return a.astype(np.float64).transpose(0, 2, 1, 3)


@pytest.mark.parametrize("T", [256, 1024])
def test_oracle_matches_reference_fixture(T):
    f = np.load(os.path.join(GOLDEN, f"refsem_T{T}.npz"))
    q, k, v, do = (bhtd(f[n]) for n in ("q", "k", "v", "do"))
    o, glob, summary = rso.fwd(q, k, v)
    # fixtures hold the reference's float64 results rounded to float32
    assert np.abs(o - bhtd(f["o"])).max() <= 1e-5
    for got, name in zip(rso.bwd(q, k, v, do), ("dq", "dk", "dv")):
        assert np.abs(got - bhtd(f[name])).max() <= 1e-5, name
    G = int(round(T ** 0.5))
    assert glob.shape[-2:] == (G, G) and summary.shape[-2:] == (G, G)
    assert np.all(glob[..., 0, :] == 0)                    # block 0 has no earlier blocks
    assert np.allclose(glob[..., 1:, :].sum(-1), 1.0)      # every other row is a softmax
    assert np.all(np.triu(np.ones((G, G), bool)) <= (glob == 0))  # strictly earlier only
    assert np.allclose(summary.sum(-1), G)                 # column sums of row-stochastic maps


def test_oracle_backward_finite_differences():
    rng = np.random.default_rng(0)
    B, H, T, D = 1, 2, 16, 4
    q, k, v, do = (rng.standard_normal((B, H, T, D)) for _ in range(4))
    dq, dk, dv = rso.bwd(q, k, v, do)
    eps = 1e-6
    for x, g in ((q, dq), (k, dk), (v, dv)):
        for idx in [(0, 0, 0, 0), (0, 1, 5, 2), (0, 0, 9, 3), (0, 1, 15, 1), (0, 0, 12, 0)]:
            xp, xm = x.copy(), x.copy()
            xp[idx] += eps
            xm[idx] -= eps
            args_p = [xp if a is x else a for a in (q, k, v)]
            args_m = [xm if a is x else a for a in (q, k, v)]
            num = ((rso.fwd(*args_p)[0] * do).sum() - (rso.fwd(*args_m)[0] * do).sum()) / (2 * eps)
            assert abs(num - g[idx]) <= 1e-6 * max(1.0, abs(num)), (idx, num, g[idx])


def test_oracle_block0_is_local_attention_and_causal():
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 1, 64, 8)) for _ in range(3))
    o, _, _ = rso.fwd(q, k, v)
    # changing the future (last block) leaves every earlier row unchanged
    k2, v2 = k.copy(), v.copy()
    k2[..., 56:, :] += 1.0
    v2[..., 56:, :] -= 2.0
    o2, _, _ = rso.fwd(q, k2, v2)
    assert np.abs(o2[..., :56, :] - o[..., :56, :]).max() == 0.0


@pytest.mark.parametrize("T", [0, 2, 15, 17, 1000])
def test_geometry_rejects_non_squares(T):
    with pytest.raises(ValueError, match="perfect square"):
        rso.geometry(T)


def test_torch_port_matches_oracle():
    """The torch restatement timed as the refsem reference arm agrees with the
    float64 oracle (which is pinned to the reference module's own outputs)."""
    import torch

    from oracle.refsem_torch_port import reference_core

    g = np.random.default_rng(5)
    q, k, v, do = (g.standard_normal((2, 3, 256, 32)) for _ in range(4))
    ro, _, _ = rso.fwd(q, k, v)
    rq, rk, rv = rso.bwd(q, k, v, do)
    tq, tk, tv = (torch.from_numpy(x).requires_grad_(True) for x in (q, k, v))
    out = reference_core(tq, tk, tv)
    (out * torch.from_numpy(do)).sum().backward()
    assert np.abs(out.detach().numpy() - ro).max() < 1e-10
    for a, r in ((tq, rq), (tk, rk), (tv, rv)):
        assert np.abs(a.grad.numpy() - r).max() < 1e-10
