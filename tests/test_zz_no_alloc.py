"""sqb_bwd_noalloc: the backward for callers that cannot allocate device memory.

Such callers (their memory belongs to another component, or their device
footprint is fixed after start-up) get the backward with the scratch held by
the library in a static device array instead of a workspace they pass.  These
tests call it through the C ABI and compare it with the regular sqb_bwd on the
same inputs, within the parity tolerances of tests/test_parity_gpu.py, on two
calls in a row (the array keeps the previous call's contents, so the second
call checks that each call clears what it needs).  This file is collected
last so that a run stopping at its first failure has run every other test.
"""

import ctypes
import math

import pytest
import torch

from llm_training_b200 import _lib
from llm_training_b200.ops import sqrt_block_backward, sqrt_block_forward

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_GRAD_REL_TOL = 1e-2


def noalloc_backward(q, k, v, o, lse, kbar, vbar, dout, block):
    B, T, H, D = q.shape
    b, _, Gc = _lib.geometry(T, block)
    dq, dk, dv = [torch.empty((B, T, H, D), dtype=q.dtype, device=q.device) for _ in range(3)]
    st = _lib.strides_array(*((t.stride(0), t.stride(1), t.stride(2))
                              for t in (q, k, v, o, dout, dq, dk, dv)))
    dtype = _lib.SQB_BF16 if q.dtype == torch.bfloat16 else _lib.SQB_F32
    rc = _lib.lib().sqb_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
        lse.data_ptr(), kbar.data_ptr() if Gc else None, vbar.data_ptr() if Gc else None,
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, T, H, D, b, st, dtype,
        1.0 / math.sqrt(D), _lib.IMPL_AUTO, torch.cuda.current_stream().cuda_stream)
    _lib.check("sqb_bwd_noalloc", rc)
    return dq, dk, dv


def close(got, ref, dtype):
    got, ref = got.float(), ref.float()
    if dtype == torch.float32:
        return (got - ref).abs().max().item() <= F32_TOL
    d = got - ref
    return ((d.abs().max() / ref.abs().max()).item() <= BF16_GRAD_REL_TOL
            and (d.norm() / ref.norm()).item() <= BF16_GRAD_REL_TOL)


@pytest.mark.parametrize("dtype,shape,block", [
    (torch.bfloat16, (2, 1024, 4, 64), 32),
    (torch.bfloat16, (1, 4096, 2, 128), None),
    (torch.bfloat16, (1, 1000, 2, 128), 128),
    # b > 128: the cross sub-tile dK / dV and reader-count regions of the scratch
    (torch.bfloat16, (1, 4096, 2, 128), 192),
    (torch.float32, (2, 256, 4, 32), 16),
])
def test_noalloc_matches_workspace_backward(dtype, shape, block):
    g = torch.Generator().manual_seed(17)
    q, k, v, do = [torch.randn(*shape, generator=g).to(dtype).cuda() for _ in range(4)]
    o, lse, kbar, vbar = sqrt_block_forward(q, k, v, block)
    ref = sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do, block)
    for _ in range(2):
        got = noalloc_backward(q, k, v, o, lse, kbar, vbar, do, block)
        torch.cuda.synchronize()
        for name, a, r in zip(("dq", "dk", "dv"), got, ref):
            assert close(a, r, dtype), name
    # no device-side failure was recorded in the library's scratch
    detail = ctypes.c_int64(-1)
    assert _lib.lib().sqb_read_status_noalloc(torch.cuda.current_stream().cuda_stream,
                                              ctypes.byref(detail)) == 0
    assert detail.value == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    # B=1, H=64, T=16384, D=128 needs ~13 MB of scratch, over the 8 MiB array
    B, T, H, D = 1, 16384, 64, 128
    assert _lib.workspace_bytes(B, T, H, D, 128) > (8 << 20)
    x = torch.empty(1, device="cuda", dtype=torch.bfloat16)
    st = _lib.strides_array(*([(T * H * D, H * D, D)] * 8))
    rc = _lib.lib().sqb_bwd_noalloc(*([x.data_ptr()] * 11), B, T, H, D, 128, st,
                                    _lib.SQB_BF16, 1.0 / math.sqrt(D), _lib.IMPL_AUTO,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 5  # SQB_ERR_WORKSPACE
