"""Generate the golden fixtures under tests/golden/.  Run where a checkout of the
reference repository is available (it is read, never modified):

    python tests/golden/make_golden.py --reference PATH_TO_REFERENCE_CHECKOUT

Fixtures written:

* ``ref_block0_T256.npz`` / ``ref_block0_T1024.npz`` - outputs of the
  reference's own registered ``sqrt_block`` module (model/custom_attention.py:138)
  run in float64 on seeded inputs, with T a perfect square so its
  ``block_geometry`` (custom_attention.py:68-79) accepts it and its block length
  sqrt(T) equals ours (16 and 32).  For block 0 the reference computes
  local[0] @ V[0] (custom_attention.py:106-109, glob row 0 == 0 at :212-213),
  which is exactly the sqrt-block operator's block 0.  The module's Wq/Wk/Wv
  are seeded random and c_proj is the identity, so the stored output is the
  attention core's.  Inputs are stored as float16 values (exact in float64).
* ``refsem_T256.npz`` / ``refsem_T1024.npz`` - the reference module's full
  attention core (all blocks, its own semantics: column-sum summaries, the G x G
  summary softmax and the fixed-weight own block, custom_attention.py:183-225 and
  _ScaledBlockCombine :82-135) and its autograd gradients, run in float64 with
  its Wq/Wk/Wv replaced by modules returning seeded leaf tensors Q, K, V and
  c_proj the identity, so the stored output and dQ/dK/dV are the core's.  They
  pin oracle/refsem_oracle.py and the CUDA reference-semantics mode.
* ``ref_metrics_schema.json`` - the key paths of the reference trainer's
  ``metrics.json`` (metrics.py:516-537: run / aggregates / train / val / _stats),
  read from the run it ships (vanilla/metrics.json); the training report of
  this repository writes the same schema.
* ``oracle_T200.npz`` - a frozen forward/backward of the oracle itself on a
  ragged case (T=200, b=16: 12 complete blocks and a partial block of 8), so
  any later change to the oracle shows up as a fixture mismatch.

The reference is imported directly as ``model.custom_attention``: going through
its registry would raise on the first lookup (model/flash_attention.py:5 has a
relative import beyond the top-level package, hit by model/attention_registry.py:103-107).
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _reference_block0(ref_root, B, H, T, D, seed):
    import torch

    sys.path.insert(0, ref_root)
    try:
        from model.custom_attention import CustomAttention  # noqa: E402
    finally:
        sys.path.pop(0)

    class Cfg:
        n_embd = H * D
        n_head = H
        block_size = T
        bias = False
        dropout = 0.0

    C = H * D
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, T, C)).astype(np.float16)
    # scale so that Q = X Wq^T has unit-variance entries
    w = (rng.standard_normal((3, C, C)) / np.sqrt(C)).astype(np.float16)
    mod = CustomAttention(Cfg()).double().eval()
    with torch.no_grad():
        mod.Wq.weight.copy_(torch.from_numpy(w[0].astype(np.float64)))
        mod.Wk.weight.copy_(torch.from_numpy(w[1].astype(np.float64)))
        mod.Wv.weight.copy_(torch.from_numpy(w[2].astype(np.float64)))
        mod.c_proj.weight.copy_(torch.eye(C, dtype=torch.float64))
        y = mod(torch.from_numpy(x.astype(np.float64))).numpy()
    L = int(round(T ** 0.5))
    return x, w, y[:, :L, :], y


def _reference_full(ref_root, B, H, T, D, seed):
    """Output and dQ/dK/dV of the reference's attention core on seeded Q/K/V/dO."""
    import torch

    sys.path.insert(0, ref_root)
    try:
        from model.custom_attention import CustomAttention  # noqa: E402
    finally:
        sys.path.pop(0)

    class Cfg:
        n_embd = H * D
        n_head = H
        block_size = T
        bias = False
        dropout = 0.0

    class Fixed(torch.nn.Module):
        """Stands in for a projection: returns a given leaf tensor."""

        def __init__(self, t):
            super().__init__()
            self.t = t

        def forward(self, x):
            return self.t

    C = H * D
    rng = np.random.default_rng(seed)
    q, k, v, do = [rng.standard_normal((B, T, H, D)).astype(np.float16) for _ in range(4)]
    mod = CustomAttention(Cfg()).double().eval()
    leaves = [torch.from_numpy(a.astype(np.float64)).reshape(B, T, C).requires_grad_()
              for a in (q, k, v)]
    mod.Wq, mod.Wk, mod.Wv = (Fixed(t) for t in leaves)
    mod.c_proj = torch.nn.Identity()
    y = mod(torch.zeros(B, T, C, dtype=torch.float64))
    y.backward(torch.from_numpy(do.astype(np.float64)).reshape(B, T, C))
    grads = [t.grad.numpy().reshape(B, T, H, D) for t in leaves]
    return q, k, v, do, y.detach().numpy().reshape(B, T, H, D), grads


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the reference checkout (read only)")
    args = ap.parse_args()
    sys.path.insert(0, REPO)
    from oracle import sqrtblock_oracle as orc

    for (B, H, T, D, seed) in [(2, 4, 256, 32, 1), (1, 2, 1024, 64, 2)]:
        x, w, y0, y = _reference_block0(args.reference, B, H, T, D, seed)
        # record how far the reference departs from the sqrt-block operator
        # after block 0 (the two are different operators there)
        xf = x.astype(np.float64)
        q, k, v = [(xf @ w[i].astype(np.float64).T).reshape(B, T, H, D).transpose(0, 2, 1, 3)
                   for i in range(3)]
        L = int(round(T ** 0.5))
        o, _ = orc.fwd_dense(q, k, v, L)
        o = o.transpose(0, 2, 1, 3).reshape(B, T, H * D)
        diff_after = float(np.abs(o[:, L:] - y[:, L:]).max())
        path = os.path.join(HERE, f"ref_block0_T{T}.npz")
        np.savez_compressed(path, x=x, w=w, y_block0=y0, shape=np.array([B, H, T, D]),
                            max_abs_diff_after_block0=np.array(diff_after))
        print(f"wrote {path}: block0 max|oracle-ref| = {np.abs(o[:, :L] - y0).max():.3e}, "
              f"after block 0 = {diff_after:.3f}")

    # state-dict keys and shapes of the reference's GPT with sqrt_block
    # attention (checkpoint compatibility: train.py:83 saves model.state_dict())
    import json

    import torch

    sys.path.insert(0, args.reference)
    try:
        import model.custom_attention  # noqa: F401  registers sqrt_block
        from model.GPT import GPT as RefGPT
    finally:
        sys.path.pop(0)
    keys = {}
    for bias in (False, True):
        class Cfg:
            block_size = 256
            vocab_size = 101
            n_layer = 2
            n_head = 4
            n_embd = 64
            dropout = 0.0
            attention = "sqrt_block"
        Cfg.bias = bias
        torch.manual_seed(0)
        try:
            m = RefGPT(Cfg())
        except ImportError:
            # the reference registry's first lookup raises after registering
            # the importable modules (attention_registry.py:101 sets
            # _discovered before model/flash_attention.py:5 fails); the
            # second lookup succeeds
            m = RefGPT(Cfg())
        keys[f"bias={bias}"] = {k: list(v.shape) for k, v in m.state_dict().items()}
    path = os.path.join(HERE, "ref_state_dict_keys.json")
    with open(path, "w") as f:
        json.dump({"config": {"block_size": 256, "vocab_size": 101, "n_layer": 2, "n_head": 4,
                              "n_embd": 64, "attention": "sqrt_block"}, "keys": keys}, f,
                  indent=1, sort_keys=True)
    print(f"wrote {path}")

    from oracle import refsem_oracle as rso

    for (B, H, T, D, seed) in [(2, 2, 256, 32, 4), (1, 1, 1024, 32, 5)]:
        q, k, v, do, y, (dq, dk, dv) = _reference_full(args.reference, B, H, T, D, seed)
        # (B, T, H, D) -> (B, H, T, D) for the oracle
        t = lambda a: a.astype(np.float64).transpose(0, 2, 1, 3)  # noqa: E731
        o_orc, _, _ = rso.fwd(t(q), t(k), t(v))
        g_orc = rso.bwd(t(q), t(k), t(v), t(do))
        err = max([np.abs(o_orc - t(y)).max()] +
                  [np.abs(a - t(b)).max() for a, b in zip(g_orc, (dq, dk, dv))])
        path = os.path.join(HERE, f"refsem_T{T}.npz")
        np.savez_compressed(path, q=q, k=k, v=v, do=do, o=y.astype(np.float32),
                            dq=dq.astype(np.float32), dk=dk.astype(np.float32),
                            dv=dv.astype(np.float32))
        print(f"wrote {path}: max|oracle - reference| = {err:.3e}")

    # key paths of the reference's metrics.json ("[]" marks a list's rows)
    def paths(x, prefix=""):
        if isinstance(x, dict):
            for k, v in x.items():
                yield f"{prefix}/{k}"
                yield from paths(v, f"{prefix}/{k}")
        elif isinstance(x, list) and x:
            yield from paths(x[0], f"{prefix}[]")

    with open(os.path.join(args.reference, "vanilla", "metrics.json")) as f:
        recorded = json.load(f)
    path = os.path.join(HERE, "ref_metrics_schema.json")
    with open(path, "w") as f:
        json.dump({"source": "vanilla/metrics.json of the reference",
                   "paths": sorted(set(paths(recorded)))}, f, indent=1)
    print(f"wrote {path}")

    B, H, T, D, b = 1, 2, 200, 32, 16
    rng = np.random.default_rng(3)
    q, k, v, do = [rng.standard_normal((B, H, T, D)).astype(np.float16) for _ in range(4)]
    o, lse = orc.fwd_dense(q, k, v, b)
    dq, dk, dv = orc.bwd_dense(q, k, v, do, b)
    path = os.path.join(HERE, "oracle_T200.npz")
    np.savez_compressed(path, q=q, k=k, v=v, do=do, b=np.array(b),
                        o=o.astype(np.float32), lse=lse.astype(np.float32),
                        dq=dq.astype(np.float32), dk=dk.astype(np.float32),
                        dv=dv.astype(np.float32))
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
