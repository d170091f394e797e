"""The custom ops' fake implementations (what torch.compile traces against),
checked on CPU under FakeTensorMode: output shapes, dtypes and the block
geometry they assume, without running a kernel."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from llm_training_b200 import ops


@pytest.mark.parametrize("T,block,Gc", [(1024, None, 32), (1000, 128, 7), (100, None, 6)])
def test_attention_fakes(T, block, Gc):
    B, H, D = 2, 4, 64
    with FakeTensorMode():
        q = torch.empty(B, T, H, D, dtype=torch.bfloat16)
        o, lse, kbar, vbar = torch.ops.sqrtblock.attention_fwd(q, q, q, block, None, "auto")
        assert o.shape == (B, T, H, D) and o.dtype == torch.bfloat16
        assert lse.shape == (B, H, T) and lse.dtype == torch.float32
        assert kbar.shape == vbar.shape == (B, H, Gc, D)
        dq, dk, dv = torch.ops.sqrtblock.attention_bwd(q, q, q, o, lse, kbar, vbar, o, block,
                                                       None, "auto")
        assert dq.shape == dk.shape == dv.shape == (B, T, H, D)
        qkv = torch.empty(B, T, 3 * H * D, dtype=torch.bfloat16)
        o2, lse2, kb2, vb2 = torch.ops.sqrtblock.attention_qkv_fwd(qkv, H, block, None, "auto")
        assert o2.shape == (B, T, H, D) and lse2.shape == (B, H, T)
        assert kb2.shape == (B, H, Gc, D)
        dqkv = torch.ops.sqrtblock.attention_qkv_bwd(qkv, o2, lse2, kb2, vb2, o2, H, block,
                                                     None, "auto")
        assert dqkv.shape == qkv.shape and dqkv.dtype == qkv.dtype


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_layernorm_fakes(bias, out):
    N, C = 64, 768
    with FakeTensorMode():
        x = torch.empty(N, C)
        h = torch.empty(N, C, dtype=torch.bfloat16)
        w = torch.empty(C)
        b = torch.empty(C) if bias else None
        y, mean, rstd = torch.ops.sqrtblock.layernorm_fwd(x, w, b, 1e-5, out)
        assert y.shape == (N, C) and y.dtype == out and mean.shape == rstd.shape == (N,)
        xo, y2, mean2, _ = torch.ops.sqrtblock.add_layernorm_fwd(x, h, w, b, 1e-5, out)
        assert xo.shape == (N, C) and xo.dtype == torch.float32 and y2.dtype == out
        dx, dh, dw, db = torch.ops.sqrtblock.add_layernorm_bwd(y2, xo, w, mean2, mean2, x,
                                                               bias, True)
        assert dx.dtype == torch.float32 and dh.shape == (N, C) and dh.dtype == torch.bfloat16
        assert dw.shape == (C,) and db.shape == ((C,) if bias else (0,))
        dx, dh, dw, db = torch.ops.sqrtblock.add_layernorm_bwd(y2, xo, w, mean2, mean2, None,
                                                               bias, False)
        assert dh.shape == (0,)


def test_fake_geometry_matches_library():
    from llm_training_b200 import _lib

    for T in (1, 15, 16, 17, 255, 256, 1000, 1024, 4097, 16384, 32768):
        for block in (None, 32, 96, 192):
            assert ops._fake_geometry(T, block) == _lib.geometry(T, block), (T, block)
