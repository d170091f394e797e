"""The CPU oracle: pinned to the reference where the operators coincide, and
cross-checked between independent restatements elsewhere."""

import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import sqrtblock_oracle as orc
from oracle.torch_port import sqrt_block_attention_ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _rand(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape)


@pytest.mark.parametrize("T,b", [(256, 16), (1024, 32), (4096, 64), (8192, 96), (16384, 128),
                                 (32768, 192), (65536, 256), (1, 16), (17, 16), (1025, 48)])
def test_default_geometry(T, b):
    assert orc.default_block(T) == b
    bb, G, Gc = orc.geometry(T)
    assert bb == b and G == math.ceil(T / b) and Gc == T // b


def test_geometry_rejects_bad_input():
    with pytest.raises(ValueError):
        orc.default_block(0)
    with pytest.raises(ValueError):
        orc.geometry(16, 0)


@pytest.mark.parametrize("T", [256, 1024])
def test_block0_matches_reference_module(T):
    """Block 0 of the operator equals the reference sqrt_block module's block 0
    (fixture made by running model/custom_attention.py in float64)."""
    f = np.load(os.path.join(GOLDEN, f"ref_block0_T{T}.npz"))
    B, H, T_, D = [int(x) for x in f["shape"]]
    assert T_ == T
    x = f["x"].astype(np.float64)
    w = f["w"].astype(np.float64)
    q, k, v = [(x @ w[i].T).reshape(B, T, H, D).transpose(0, 2, 1, 3) for i in range(3)]
    L = math.isqrt(T)
    assert orc.default_block(T) == L
    o, _ = orc.fwd_dense(q, k, v, L)
    o = o.transpose(0, 2, 1, 3).reshape(B, T, H * D)
    np.testing.assert_allclose(o[:, :L], f["y_block0"], rtol=0, atol=1e-12)
    # the reference is a different operator after block 0 (recorded, not a target)
    assert float(f["max_abs_diff_after_block0"]) > 0.1


def test_frozen_oracle_fixture():
    f = np.load(os.path.join(GOLDEN, "oracle_T200.npz"))
    b = int(f["b"])
    o, lse = orc.fwd_blockwise(f["q"], f["k"], f["v"], b)
    dq, dk, dv = orc.bwd_blockwise(f["q"], f["k"], f["v"], f["do"], b)
    for name, got in [("o", o), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)]:
        np.testing.assert_allclose(got, f[name], rtol=0, atol=2e-6, err_msg=name)


@pytest.mark.parametrize("B,H,T,D,b", [(2, 4, 256, 32, 16), (1, 2, 200, 16, 16),
                                       (1, 1, 50, 8, 16), (1, 1, 7, 8, 16), (1, 2, 300, 8, 96)])
def test_dense_blockwise_torch_agree(B, H, T, D, b):
    q, k, v, do = [_rand((B, H, T, D), s) for s in range(4)]
    o1, l1 = orc.fwd_dense(q, k, v, b)
    o2, l2 = orc.fwd_blockwise(q, k, v, b)
    np.testing.assert_allclose(o1, o2, atol=1e-12)
    np.testing.assert_allclose(l1, l2, atol=1e-12)
    g1 = orc.bwd_dense(q, k, v, do, b)
    g2 = orc.bwd_blockwise(q, k, v, do, b)
    for a, c in zip(g1, g2):
        np.testing.assert_allclose(a, c, atol=1e-11)
    tq, tk, tv = [torch.tensor(a, requires_grad=True) for a in (q, k, v)]
    o3, l3 = sqrt_block_attention_ref(tq, tk, tv, b)
    (o3 * torch.tensor(do)).sum().backward()
    np.testing.assert_allclose(o3.detach().numpy(), o1, atol=1e-12)
    np.testing.assert_allclose(l3.detach().numpy(), l1, atol=1e-12)
    for t, g in zip((tq, tk, tv), g1):
        np.testing.assert_allclose(t.grad.numpy(), g, atol=1e-11)


def test_gradcheck_torch_port():
    g = torch.Generator().manual_seed(0)
    q, k, v = [torch.randn(1, 2, 40, 4, generator=g, dtype=torch.float64, requires_grad=True)
               for _ in range(3)]
    assert torch.autograd.gradcheck(lambda a, c, d: sqrt_block_attention_ref(a, c, d, 16)[0],
                                    (q, k, v), eps=1e-6, atol=1e-6)


def test_analytic_backward_matches_finite_differences():
    q, k, v, do = [_rand((1, 1, 37, 4), s + 10) for s in range(4)]
    dq, dk, dv = orc.bwd_dense(q, k, v, do, 16)
    eps = 1e-6
    rng = np.random.default_rng(0)
    for arr, grad in ((q, dq), (k, dk), (v, dv)):
        for _ in range(6):
            idx = tuple(rng.integers(0, s) for s in arr.shape)
            a1, a2 = arr.copy(), arr.copy()
            a1[idx] += eps
            a2[idx] -= eps
            args1 = [a1 if x is arr else x for x in (q, k, v)]
            args2 = [a2 if x is arr else x for x in (q, k, v)]
            f1 = (orc.fwd_dense(*args1, 16)[0] * do).sum()
            f2 = (orc.fwd_dense(*args2, 16)[0] * do).sum()
            assert abs((f1 - f2) / (2 * eps) - grad[idx]) < 1e-6


def test_causality():
    """Perturbing tokens >= t0 leaves every output before t0 bit-identical."""
    T, b = 300, 32
    q, k, v = [_rand((1, 2, T, 16), s) for s in range(3)]
    o, _ = orc.fwd_blockwise(q, k, v, b)
    for t0 in (1, 31, 32, 33, 100, 256, 299):
        q2, k2, v2 = q.copy(), k.copy(), v.copy()
        for a in (q2, k2, v2):
            a[..., t0:, :] += 3.0
        o2, _ = orc.fwd_blockwise(q2, k2, v2, b)
        assert np.array_equal(o[..., :t0, :], o2[..., :t0, :])


def test_block0_is_causal_attention():
    T, b = 64, 32
    q, k, v = [_rand((2, 3, T, 8), s) for s in range(3)]
    o, _ = orc.fwd_dense(q, k, v, b)
    s = np.einsum("...td,...kd->...tk", q[..., :b, :], k[..., :b, :]) / math.sqrt(8)
    s = np.where(np.tril(np.ones((b, b), bool)), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    np.testing.assert_allclose(o[..., :b, :], p @ v[..., :b, :], atol=1e-12)


def test_partial_last_block_has_no_summary():
    """T=200, b=16: 12 complete blocks; the 8-row tail sees 12 summaries and
    contributes to none, and its keys only receive in-block gradient."""
    T, b = 200, 16
    q, k, v, do = [_rand((1, 1, T, 8), s) for s in range(4)]
    assert orc.pool(k, b).shape[-2] == 12
    dq, dk, dv = orc.bwd_dense(q, k, v, do, b)
    # zero the tail's upstream gradient: its K/V gradient must vanish
    do2 = do.copy()
    do2[..., 192:, :] = 0
    _, dk2, dv2 = orc.bwd_dense(q, k, v, do2, b)
    assert np.abs(dk2[..., 192:, :]).max() == 0 and np.abs(dv2[..., 192:, :]).max() == 0


def test_work_formulas_match_published_table():
    # B=1, H=16, T=16384, D=128, b=128: 60.13 GFLOP and 807.4 MB
    assert orc.algorithmic_flops(1, 16, 16384, 128, 128) == 60129542144
    assert orc.algorithmic_bytes(1, 16, 16384, 128, 2) == 807403520
    assert orc.pairs(256, 16) == sum((t % 16) + 1 + t // 16 for t in range(256))


def test_reference_state_dict_fixture_is_well_formed():
    d = json.load(open(os.path.join(GOLDEN, "ref_state_dict_keys.json")))
    for keys in d["keys"].values():
        assert any(k.endswith("attn.Wq.weight") for k in keys)
