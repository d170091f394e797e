"""Fused LayerNorm of the training caller (include/sqb_train.h).

CPU: argument rejection without touching a device.  GPU: output and the three
gradients against ``F.layer_norm`` in fp32 (with and without a bias, fp32 or
bf16 output, fp32 or bf16 upstream gradient, row counts that do not fill the
last CTA), and the GPT caller's LayerNorm module against nn.LayerNorm."""

import ctypes

import pytest
import torch
import torch.nn.functional as F

from llm_training_b200 import _lib

ERR_ARG, ERR_UNSUPPORTED, ERR_WORKSPACE = 1, 4, 5  # include/sqrtblock.h


def test_rejects_bad_arguments_without_a_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    assert lib.sqb_layernorm_fwd(None, p, None, p, 0, p, p, 4, 128, 1e-5, None) == ERR_ARG
    assert lib.sqb_layernorm_fwd(p, p, None, p, 0, p, p, 4, 100, 1e-5, None) == ERR_UNSUPPORTED
    assert lib.sqb_layernorm_fwd(p, p, None, p, 0, p, p, 4, 2048, 1e-5, None) == ERR_UNSUPPORTED
    assert lib.sqb_layernorm_workspace_bytes(16384, 768) > 0
    assert lib.sqb_layernorm_bwd(p, 0, p, p, p, p, p, p, None, p, 16, 4, 128,
                                 None) == ERR_WORKSPACE


@pytest.mark.gpu
@pytest.mark.parametrize("N,C,bias,out,dyt", [
    (1000, 768, False, torch.float32, torch.float32),
    (1000, 768, True, torch.bfloat16, torch.bfloat16),
    (4097, 1024, False, torch.bfloat16, torch.bfloat16),
    (3, 128, True, torch.float32, torch.float32),
    (5003, 384, True, torch.bfloat16, torch.float32),
])
def test_matches_torch_layer_norm(N, C, bias, out, dyt):
    from llm_training_b200.ops import layer_norm

    g = torch.Generator().manual_seed(N + C)
    x = (torch.randn(N, C, generator=g) * 2 + 0.5).cuda()
    w = (1 + 0.1 * torch.randn(C, generator=g)).cuda()
    b = (0.1 * torch.randn(C, generator=g)).cuda() if bias else None
    dy = torch.randn(N, C, generator=g).to(dyt).cuda()
    xs, ws = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    bs = b.clone().requires_grad_(True) if bias else None
    y = layer_norm(xs, ws, bs, 1e-5, out)
    assert y.dtype == out
    y.backward(dy.to(out))
    xr, wr = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    br = b.clone().requires_grad_(True) if bias else None
    yr = F.layer_norm(xr, (C,), wr, br, 1e-5)
    yr.backward(dy.to(out).float())
    if out == torch.float32:
        torch.testing.assert_close(y, yr, rtol=1e-5, atol=1e-5)
    else:
        torch.testing.assert_close(y.float(), yr, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(xs.grad, xr.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ws.grad, wr.grad, rtol=1e-4, atol=1e-3)
    if bias:
        torch.testing.assert_close(bs.grad, br.grad, rtol=1e-4, atol=1e-3)


@pytest.mark.gpu
def test_gpt_layernorm_module_matches_nn_layernorm_under_autocast():
    from llm_training_b200.model.gpt import LayerNorm

    torch.manual_seed(0)
    m = LayerNorm(768, bias=False).cuda()
    with torch.no_grad():
        m.ln.weight.add_(0.1 * torch.randn(768, device="cuda"))
    x = torch.randn(8, 64, 768, device="cuda", requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
        y_ref = m.ln(x)  # nn.LayerNorm: fp32 under autocast
    assert y.dtype == torch.bfloat16 and y_ref.dtype == torch.float32
    torch.testing.assert_close(y.float(), y_ref.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
    (gx,) = torch.autograd.grad(y.float().sum(), x)
    (gx_ref,) = torch.autograd.grad(y_ref.to(torch.bfloat16).float().sum(), x)
    torch.testing.assert_close(gx, gx_ref, rtol=1e-4, atol=1e-4)


def test_add_variant_rejects_bad_arguments_without_a_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    # no h, or h without an x_out destination
    assert lib.sqb_add_layernorm_fwd(p, None, 0, p, p, None, p, 0, p, p, 4, 128, 1e-5,
                                     None) == ERR_ARG
    assert lib.sqb_add_layernorm_fwd(p, p, 0, None, p, None, p, 0, p, p, 4, 128, 1e-5,
                                     None) == ERR_ARG
    assert lib.sqb_add_layernorm_bwd(p, 0, p, p, p, p, None, p, None, p, None, p, 16, 4, 128,
                                     None) == ERR_WORKSPACE


@pytest.mark.gpu
@pytest.mark.parametrize("N,C,bias,ht,out,with_res", [
    (1000, 768, False, torch.bfloat16, torch.bfloat16, True),
    (4097, 1024, True, torch.bfloat16, torch.bfloat16, False),
    (3, 128, True, torch.float32, torch.float32, True),
    (5003, 384, False, torch.float32, torch.bfloat16, True),
])
def test_add_layer_norm_matches_add_then_layer_norm(N, C, bias, ht, out, with_res):
    """(x + h, LayerNorm(x + h)) and its gradients against torch's add and
    F.layer_norm in fp32; the residual output's own downstream gradient (with_res)
    joins the LayerNorm's input gradient."""
    from llm_training_b200.ops import add_layer_norm

    g = torch.Generator().manual_seed(N + 7 * C)
    x = (torch.randn(N, C, generator=g) * 2 + 0.5).cuda()
    h = torch.randn(N, C, generator=g).to(ht).cuda()
    w = (1 + 0.1 * torch.randn(C, generator=g)).cuda()
    b = (0.1 * torch.randn(C, generator=g)).cuda() if bias else None
    dy = torch.randn(N, C, generator=g).to(out).cuda()
    dxo = torch.randn(N, C, generator=g).cuda()

    def leaves():
        return (x.clone().requires_grad_(True), h.clone().requires_grad_(True),
                w.clone().requires_grad_(True), b.clone().requires_grad_(True) if bias else None)

    xs, hs, ws, bs = leaves()
    xo, y = add_layer_norm(xs, hs, ws, bs, 1e-5, out)
    assert xo.dtype == torch.float32 and y.dtype == out
    outs, grads = ((xo, y), (dxo, dy)) if with_res else ((y,), (dy,))
    torch.autograd.backward(outs, grads)
    xr, hr, wr, br = leaves()
    xor = xr + hr
    yr = F.layer_norm(xor, (C,), wr, br, 1e-5)
    outs_r, grads_r = ((xor, yr), (dxo, dy.float())) if with_res else ((yr,), (dy.float(),))
    torch.autograd.backward(outs_r, grads_r)
    torch.testing.assert_close(xo, xor, rtol=0, atol=0)  # the same fp32 sum
    if out == torch.float32:
        torch.testing.assert_close(y, yr, rtol=1e-5, atol=1e-5)
    else:
        torch.testing.assert_close(y.float(), yr, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(xs.grad, xr.grad, rtol=1e-4, atol=1e-4)
    assert hs.grad.dtype == ht
    torch.testing.assert_close(hs.grad.float(), hr.grad.float(),
                               rtol=1e-2 if ht == torch.bfloat16 else 1e-4,
                               atol=1e-2 if ht == torch.bfloat16 else 1e-4)
    torch.testing.assert_close(ws.grad, wr.grad, rtol=1e-4, atol=1e-3)
    if bias:
        torch.testing.assert_close(bs.grad, br.grad, rtol=1e-4, atol=1e-3)
