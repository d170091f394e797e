"""Fused token cross-entropy of the training caller (include/sqb_train.h).

CPU: the library exports and binds every symbol the header declares and rejects
bad arguments before touching a device.  GPU: value and gradient against
``F.cross_entropy`` in fp32 on the same logits (bf16 and fp32 inputs, ignored
targets, -inf padding columns, a row pitch wider than the vocabulary, and an odd
vocabulary that takes the scalar-load path)."""

import ctypes
import os
import re

import pytest
import torch
import torch.nn.functional as F

from llm_training_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "sqb_train.h")
ERR_ARG, ERR_DTYPE = 1, 2  # SQB_ERR_ARG, SQB_ERR_DTYPE (include/sqrtblock.h)


def test_library_exports_every_training_symbol():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    syms = sorted(set(re.findall(r"\b(sqb_[a-z_]+)\s*\(", text)))
    assert syms == sorted(_lib.TRAIN_SIGNATURES)
    lib = _lib.lib()
    for s in syms:
        assert hasattr(lib, s), s


def test_rejects_bad_arguments_without_a_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    assert lib.sqb_xent_fwd(None, p, p, p, 4, 8, 8, _lib.SQB_BF16, None) == ERR_ARG
    assert lib.sqb_xent_fwd(p, p, p, p, 4, 8, 7, _lib.SQB_BF16, None) == ERR_ARG
    assert lib.sqb_xent_fwd(p, p, p, p, 0, 8, 8, _lib.SQB_BF16, None) == ERR_ARG
    assert lib.sqb_xent_fwd(p, p, p, p, 4, 8, 8, 7, None) == ERR_DTYPE
    assert lib.sqb_xent_bwd(p, p, p, None, p, 4, 8, 8, _lib.SQB_F32, None) == ERR_ARG
    assert lib.sqb_xent_bwd(p, p, p, p, p, 4, 8, 8, 9, None) == ERR_DTYPE


def _case(N, V, dtype, pad=0, pitch=0, ignore=0, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, V + pad, generator=g) * 3
    if pad:
        x[:, V:] = float("-inf")
    t = torch.randint(0, V, (N,), generator=g)
    if ignore:
        t[torch.randperm(N, generator=g)[:ignore]] = -100
    x = x.to(dtype).cuda()
    if pitch:  # rows of a wider buffer: row stride > V + pad
        buf = torch.zeros(N, V + pad + pitch, dtype=dtype, device="cuda")
        buf[:, :V + pad] = x
        x = buf[:, :V + pad]
    return x, t.cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("N,V,dtype,pad,pitch,ignore", [
    (257, 1000, torch.bfloat16, 0, 0, 0),
    (257, 1000, torch.float32, 0, 0, 7),
    (300, 1000, torch.bfloat16, 24, 0, 0),   # -inf padding to 1024 columns
    (64, 997, torch.bfloat16, 0, 0, 3),      # odd vocabulary: scalar loads
    (64, 512, torch.bfloat16, 0, 40, 0),     # row pitch 552 > V
    (33, 50257, torch.bfloat16, 47, 0, 0),   # GPT-2 vocabulary padded to 50304
])
def test_matches_torch_cross_entropy(N, V, dtype, pad, pitch, ignore):
    from llm_training_b200.ops import cross_entropy

    x, t = _case(N, V, dtype, pad, pitch, ignore)
    a = x.detach().clone().requires_grad_(True) if pitch == 0 else x.detach().requires_grad_(True)
    loss = cross_entropy(a, t)
    loss.backward(torch.tensor(2.0, device="cuda"))
    ref_x = x.detach().float().requires_grad_(True)
    ref = F.cross_entropy(ref_x, t)
    ref.backward(torch.tensor(2.0, device="cuda"))
    torch.testing.assert_close(loss, ref, rtol=1e-5, atol=1e-5)
    gref = ref_x.grad
    scale = float(gref.abs().max())
    # the gradient is written in the logits' dtype (bf16 rounds: rtol 1e-2)
    torch.testing.assert_close(a.grad.float(), gref, rtol=1e-2, atol=1e-3 * scale)
    if pad:
        assert torch.count_nonzero(a.grad[:, V:]) == 0
