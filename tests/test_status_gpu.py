"""Device-side failure detection on the GPU, without a GPU fault.

A bounded wait is made to run out on purpose: one backward work tile's
summary-gradient counter is seeded so that the publisher's increment never
brings it to the launch epoch, so the earlier tiles of that (batch, head)
wait for it until the wait budget (shortened to 20 ms through the workspace)
runs out.  Nothing hangs: the wait gives up, records SQB_ERR_TIMEOUT, the
launch runs to its end with wrong values for the affected blocks, and its
last CTA posts the failure to the host-mapped mailbox.  The tests check that
the failure is reported - by sqb_read_status, by the mailbox without a
synchronize, and by the op's non-blocking check, which raises - and that the
next call on a re-zeroed workspace is correct again.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from llm_training_b200 import _lib, ops

pytestmark = pytest.mark.gpu

SQB_ERR_TIMEOUT = 7
BF16_GRAD_REL_TOL = 1e-2
B, T, H, D = 1, 4096, 2, 128   # b = 64: 32 work tiles of 128 rows per (batch, head)


def _bwd_counter_index(B_, T_, H_, D_, b, bh, s):
    """int32 index of the backward counter of work tile s of (batch*head) bh in
    the workspace: control block (64 words), forward flags, backward flags, each
    region 256-byte aligned and B*H*(ceil(T/16) + ceil(T/b)) words long (the
    workspace layout of csrc/sqb_internal.cuh)."""
    per_seq = -(-T_ // 16) + -(-T_ // b)
    flags_fwd = 256
    flags_bwd = (flags_fwd + B_ * H_ * per_seq * 4 + 255) // 256 * 256
    return flags_bwd // 4 + bh * per_seq + s


def _epoch(ws):
    return int(ws.view(torch.int32)[8].item())  # control word 8: backward launch epoch


def _inputs(seed=23):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).cuda() for _ in range(4)]


def _close(got, ref):
    d = got.float() - ref.float()
    return ((d.abs().max() / ref.float().abs().max()).item() <= BF16_GRAD_REL_TOL
            and (d.norm() / ref.float().norm()).item() <= BF16_GRAD_REL_TOL)


def _capi_bwd(q, k, v, o, lse, kbar, vbar, do, ws):
    b, _, _ = _lib.geometry(T)
    dq, dk, dv = [torch.empty_like(q) for _ in range(3)]
    st = _lib.strides_array(*((t.stride(0), t.stride(1), t.stride(2))
                              for t in (q, k, v, o, do, dq, dk, dv)))
    rc = _lib.lib().sqb_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                            do.data_ptr(), lse.data_ptr(), kbar.data_ptr(), vbar.data_ptr(),
                            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, T, H, D, b, st,
                            _lib.SQB_BF16, 1.0 / math.sqrt(D), _lib.IMPL_TCGEN05,
                            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    _lib.check("sqb_bwd", rc)
    return dq, dk, dv


def test_timed_out_wait_is_reported_through_the_c_abi():
    q, k, v, do = _inputs()
    o, lse, kbar, vbar = ops.sqrt_block_forward(q, k, v)
    ref = ops.sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do)
    b, _, _ = _lib.geometry(T)
    ws = torch.zeros(_lib.workspace_bytes(B, T, H, D, b), dtype=torch.uint8, device="cuda")
    mailbox = torch.zeros(2, dtype=torch.int32, pin_memory=True)
    stream = torch.cuda.current_stream().cuda_stream
    lib = _lib.lib()
    _lib.check("sqb_attach_status", lib.sqb_attach_status(ws.data_ptr(), mailbox.data_ptr(),
                                                          20000, stream))
    # tile 5 of head 0 never publishes: tiles 0-4 of head 0 wait for it
    ws.view(torch.int32)[_bwd_counter_index(B, T, H, D, b, 0, 5)] = _epoch(ws) - 1
    _capi_bwd(q, k, v, o, lse, kbar, vbar, do, ws)
    torch.cuda.synchronize()
    assert int(mailbox[0]) == SQB_ERR_TIMEOUT          # posted without a synchronize
    detail = ctypes.c_int64()
    assert lib.sqb_read_status(ws.data_ptr(), stream, ctypes.byref(detail)) == SQB_ERR_TIMEOUT
    assert detail.value == int(mailbox[1]) & 0xFFFFFFFF
    # the work tile index that gave up: a tile of head 0 before tile 5
    n = detail.value
    ntiles = T // 128
    assert n % (B * H) == 0 and ntiles - 1 - n // (B * H) < 5
    assert lib.sqb_read_status(ws.data_ptr(), stream, None) == 0   # cleared
    # zeroed again, the workspace gives correct results
    ws.zero_()
    mailbox.zero_()
    _lib.check("sqb_attach_status", lib.sqb_attach_status(ws.data_ptr(), mailbox.data_ptr(), 0,
                                                          stream))
    got = _capi_bwd(q, k, v, o, lse, kbar, vbar, do, ws)
    torch.cuda.synchronize()
    assert int(mailbox[0]) == 0
    for name, a, r in zip(("dq", "dk", "dv"), got, ref):
        assert _close(a, r), name


def test_op_raises_on_a_posted_failure_and_recovers():
    q, k, v, do = _inputs(29)
    o, lse, kbar, vbar = ops.sqrt_block_forward(q, k, v)
    ref = ops.sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do)
    torch.cuda.synchronize()
    b, _, _ = _lib.geometry(T)
    ws = ops._workspace(q.device, (B, T, H, D, b))
    ops.set_wait_budget_us(20000)
    try:
        ws.view(torch.int32)[_bwd_counter_index(B, T, H, D, b, 1, 9)] = _epoch(ws) - 1
        ops.sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do)   # launches; fails on device
        torch.cuda.synchronize()
        with pytest.raises(_lib.SqrtBlockError) as err:
            ops.check_status()                                     # no synchronize needed
        assert err.value.code == SQB_ERR_TIMEOUT
        ops.check_status()                                         # reported once, then reset
    finally:
        ops.set_wait_budget_us(0)
    got = ops.sqrt_block_backward(q, k, v, o, lse, kbar, vbar, do)
    torch.cuda.synchronize()
    ops.check_status()
    assert ops.read_status() == 0
    for name, a, r in zip(("dq", "dk", "dv"), got, ref):
        assert _close(a, r), name


def test_trainer_step_checks_the_mailboxes():
    """Trainer.step raises once a previous step's kernel posted a failure."""
    from llm_training_b200.config import ModelConfig
    from llm_training_b200.train import Trainer, synthetic_batch

    cfg = ModelConfig(n_layer=1, n_head=2, n_embd=256, block_size=4096, vocab_size=512,
                      bias=False)
    dev = torch.device("cuda", torch.cuda.current_device())
    tr = Trainer(cfg, dev)
    x, y = synthetic_batch(torch.Generator().manual_seed(0), 1, 4096, 512, dev)
    tr.step(x, y)
    torch.cuda.synchronize()
    key = next(k for k in ops._mailbox_words if k[1:] == (1, 4096, 2, 128, 64))
    ops._mailboxes[key][1] = 0x5        # as the last CTA of a failed launch posts them
    ops._mailboxes[key][0] = SQB_ERR_TIMEOUT
    with pytest.raises(_lib.SqrtBlockError):
        tr.step(x, y)
    loss, _ = tr.step(x, y)             # the workspace was reset: steps run again
    assert np.isfinite(float(loss))
