"""PyTorch entry points of the sqrt-block attention CUDA library.

``sqrt_block_attention(q, k, v)`` takes (B, T, H, D) CUDA views - exactly the
``Linear(X).view(B, T, H, D)`` layout the plugin module produces - and returns
O in the same (B, T, H, D) layout, differentiable through the library's
backward.  PyTorch only supplies device memory, the current stream and
autograd bookkeeping; all attention math runs in libsqrtblock.so.
"""

from __future__ import annotations

import math
import warnings
import threading
from typing import Optional

import torch

from . import _lib

__all__ = ["sqrt_block_attention", "sqrt_block_forward", "sqrt_block_backward", "read_status",
           "check_status", "set_wait_budget_us",
           "block_geometry", "reference_attention", "reference_forward", "reference_backward",
           "cross_entropy", "layer_norm", "layer_norm_supported"]

_DTYPES = {torch.float32: _lib.SQB_F32, torch.bfloat16: _lib.SQB_BF16}

_ws_lock = threading.Lock()
_workspaces: dict[tuple, torch.Tensor] = {}
# per workspace: two page-locked int32 words (status, detail) the kernels post a
# device-side failure to; polled without synchronizing
_mailboxes: dict[tuple, torch.Tensor] = {}
_mailbox_words: dict[tuple, "object"] = {}  # numpy views of the same words (cheap reads)
_wait_budget_us = 0  # 0 = the library default (2 s)


def block_geometry(T: int, block: int | None = None):
    """(b, G, Gc): block length, blocks, complete blocks for T tokens."""
    return _lib.geometry(T, block)


def _attach(key) -> None:
    ws, mb = _workspaces[key], _mailboxes[key]
    stream = torch.cuda.current_stream(ws.device).cuda_stream
    _lib.check("sqb_attach_status", _lib.lib().sqb_attach_status(
        ws.data_ptr(), mb.data_ptr(), _wait_budget_us, stream))


def _workspace(device: torch.device, shape: tuple) -> torch.Tensor:
    """Zero-initialised scratch for one (B, T, H, D, b) problem on one device.

    The kernels keep it clean between calls (flags are epoch-stamped and the
    summary-gradient accumulators end every call at zero), so it is zeroed
    only when allocated, and again after a device-side failure.  The region
    layout depends on the problem shape, hence one workspace per shape.  Calls
    on one device must share one stream.  Each workspace has a page-locked
    mailbox the kernels post a device-side failure to (``check_status``).
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx,) + tuple(int(x) for x in shape)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None:
            nbytes = _lib.workspace_bytes(*shape)
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
            _mailboxes[key] = torch.zeros(2, dtype=torch.int32, pin_memory=True)
            _mailbox_words[key] = _mailboxes[key].numpy()
            _attach(key)
        return ws


def _reset(key) -> None:
    """Zero a workspace (and its mailbox) after a device-side failure."""
    _workspaces[key].zero_()
    _mailboxes[key].zero_()
    _attach(key)


def check_status(device=None) -> None:
    """Raise ``SqrtBlockError`` (code SQB_ERR_TIMEOUT) if a kernel launched on
    ``device`` (default: every device) posted a device-side failure - a
    bounded wait that gave up, which leaves that call's outputs invalid.

    Never synchronizes: it reads the page-locked mailboxes the kernels write
    when they finish, so it reports failures of calls that have completed on
    the GPU by the time it runs (a call still in flight is reported by a later
    check).  Every op of this module runs it on entry, and the GPT trainer
    once per step.  The failed workspace is zeroed again before raising, so
    calls after the error compute correct results.
    """
    idx = None
    if device is not None:
        idx = device if isinstance(device, int) else (
            device.index if device.index is not None else torch.cuda.current_device())
    for key, mb in list(_mailbox_words.items()):
        if mb[0] == 0 or (idx is not None and key[0] != idx):
            continue
        code, detail = int(mb[0]), int(mb[1]) & 0xFFFFFFFF
        with _ws_lock:
            _reset(key)
        raise _lib.SqrtBlockError(
            "sqrt-block attention", code,
            f"{_lib.lib().sqb_strerror(code).decode()} in an earlier call on device {key[0]} "
            f"(problem (B, T, H, D, b) = {key[1:]}, detail {detail:#x}); that call's outputs "
            "are invalid, and its workspace has been reset")


def set_wait_budget_us(microseconds: int) -> None:
    """Budget of the kernels' waits on other work tiles (0 = the library
    default of 2 s), for every workspace of this process."""
    global _wait_budget_us
    _wait_budget_us = int(microseconds)
    with _ws_lock:
        for key in list(_workspaces):
            with torch.cuda.device(key[0]):
                _attach(key)


def _strides(t: torch.Tensor):
    return (t.stride(0), t.stride(1), t.stride(2))


def _prep(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"sqrt_block_attention: {name} must be a CUDA tensor "
                           "(the op has no CPU implementation)")
    if t.dim() != 4:
        raise ValueError(f"sqrt_block_attention: {name} must be (B, T, H, D), got {tuple(t.shape)}")
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def _impl_code(impl: str) -> int:
    try:
        return _lib.IMPLS[impl]
    except KeyError:
        raise ValueError(f"impl must be one of {sorted(_lib.IMPLS)}, got {impl!r}") from None


_simt_warned = False


def _warn_simt_once():
    """float32 inputs run on the CUDA-core kernels (the tensor-core kernels take
    bfloat16): correct, but far slower.  Said once per process."""
    global _simt_warned
    if not _simt_warned:
        _simt_warned = True
        warnings.warn("sqrt_block_attention: float32 inputs run on the CUDA-core (SIMT) "
                      "kernels, tens of times slower than the bfloat16 tensor-core kernels; "
                      "cast q/k/v to bfloat16 or run under torch.autocast(dtype=torch.bfloat16)",
                      RuntimeWarning, stacklevel=3)


def sqrt_block_forward(q, k, v, block=None, scale=None, impl="auto"):
    """Forward only -> (o, lse, kbar, vbar).

    q, k, v: (B, T, H, D) float32 or bfloat16 CUDA views (unit stride on D).
    o: (B, T, H, D) contiguous; lse: (B, H, T) fp32; kbar/vbar: (B, H, Gc, D).
    """
    q, k, v = _prep(q, "q"), _prep(k, "k"), _prep(v, "v")
    if not (q.shape == k.shape == v.shape):
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    if q.dtype not in _DTYPES:
        raise TypeError(f"sqrt_block_attention supports float32 and bfloat16, got {q.dtype}")
    B, T, H, D = q.shape
    b, G, Gc = _lib.geometry(T, block)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = q.device
    if _mailbox_words:
        check_status(dev)
    if impl == "auto" and q.dtype == torch.float32:
        _warn_simt_once()
    o = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=dev)
    kbar = torch.empty((B, H, Gc, D), dtype=q.dtype, device=dev)
    vbar = torch.empty((B, H, Gc, D), dtype=q.dtype, device=dev)
    ws = _workspace(dev, (B, T, H, D, b))
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = _lib.strides_array(_strides(q), _strides(k), _strides(v), _strides(o))
    rc = _lib.lib().sqb_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                            lse.data_ptr(), kbar.data_ptr() if Gc else None,
                            vbar.data_ptr() if Gc else None, B, T, H, D, b, st,
                            _DTYPES[q.dtype], float(scale), _impl_code(impl), ws.data_ptr(),
                            ws.numel(), stream)
    _lib.check("sqb_fwd", rc)
    return o, lse, kbar, vbar


def sqrt_block_backward(q, k, v, o, lse, kbar, vbar, dout, block=None, scale=None,
                        impl="auto", out=None):
    """Backward from saved forward outputs -> (dq, dk, dv), each (B, T, H, D).
    ``out``: three (B, T, H, D) views (unit stride on D) to write them into, e.g.
    the thirds of one packed (B, T, 3C) gradient."""
    q, k, v, o = _prep(q, "q"), _prep(k, "k"), _prep(v, "v"), _prep(o, "o")
    dout = _prep(dout, "dout")
    if dout.dtype != q.dtype:
        dout = dout.to(q.dtype)
    B, T, H, D = q.shape
    b, G, Gc = _lib.geometry(T, block)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = q.device
    if _mailbox_words:
        check_status(dev)
    if out is not None:
        dq, dk, dv = out
        for t in out:
            if (t.shape != (B, T, H, D) or t.dtype != q.dtype or t.device != dev
                    or t.stride(-1) != 1):
                raise ValueError("out must be three (B, T, H, D) tensors of q's dtype and "
                                 "device with unit stride on D")
    else:
        dq = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
        dk = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
        dv = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
    ws = _workspace(dev, (B, T, H, D, b))
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = _lib.strides_array(*(_strides(t) for t in (q, k, v, o, dout, dq, dk, dv)))
    lse = lse.contiguous()
    rc = _lib.lib().sqb_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                            dout.data_ptr(), lse.data_ptr(),
                            kbar.data_ptr() if Gc else None, vbar.data_ptr() if Gc else None,
                            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, T, H, D, b, st,
                            _DTYPES[q.dtype], float(scale), _impl_code(impl), ws.data_ptr(),
                            ws.numel(), stream)
    _lib.check("sqb_bwd", rc)
    return dq, dk, dv


def read_status(device=None) -> int:
    """Synchronize and return (then clear) the first device-side status
    recorded in any workspace of the device (0 = ok); a workspace that
    recorded a failure is zeroed again.  ``check_status`` is the
    non-synchronizing check."""
    idx = device if isinstance(device, int) else (
        device.index if device is not None and device.index is not None
        else torch.cuda.current_device())
    dev = torch.device("cuda", idx)
    stream = torch.cuda.current_stream(dev).cuda_stream
    status = _lib.SQB_OK
    for key, ws in list(_workspaces.items()):
        if key[0] != idx:
            continue
        detail = _lib.ctypes.c_int64()
        rc = _lib.lib().sqb_read_status(ws.data_ptr(), stream, _lib.ctypes.byref(detail))
        if rc != _lib.SQB_OK:
            if status == _lib.SQB_OK:
                status = rc
            with _ws_lock:
                _reset(key)
    return status


# ---- custom ops: the boundary as torch.library operators ----------------------
# The op is registered with torch.library (a fake implementation for tracing,
# autograd through the library's backward), so torch.compile - the reference
# trainer's default (train.py:28-30, :370) - traces a model using it as one
# opaque node per call instead of breaking the graph at every layer.


def _fake_geometry(T, block):
    # pure-Python twin of the library's sqb_geometry (b = round_up(ceil(sqrt(T)), 16))
    T = int(T)
    b = int(block) if block else (math.isqrt(T - 1) + 1 + 15) // 16 * 16
    return b, -(-T // b), T // b


@torch.library.custom_op("sqrtblock::attention_fwd", mutates_args=())
def _attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block: Optional[int],
                   scale: Optional[float], impl: str
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return sqrt_block_forward(q, k, v, block, scale, impl)


@_attention_fwd.register_fake
def _(q, k, v, block, scale, impl):
    B, T, H, D = q.shape
    _, _, Gc = _fake_geometry(T, block)
    return (q.new_empty((B, T, H, D)), q.new_empty((B, H, T), dtype=torch.float32),
            q.new_empty((B, H, Gc, D)), q.new_empty((B, H, Gc, D)))


@torch.library.custom_op("sqrtblock::attention_bwd", mutates_args=())
def _attention_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                   lse: torch.Tensor, kbar: torch.Tensor, vbar: torch.Tensor,
                   dout: torch.Tensor, block: Optional[int], scale: Optional[float], impl: str
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return sqrt_block_backward(q, k, v, o, lse, kbar, vbar, dout, block, scale, impl)


@_attention_bwd.register_fake
def _(q, k, v, o, lse, kbar, vbar, dout, block, scale, impl):
    return tuple(q.new_empty(q.shape) for _ in range(3))


def _attention_setup(ctx, inputs, output):
    q, k, v, block, scale, impl = inputs
    o, lse, kbar, vbar = output
    ctx.save_for_backward(q, k, v, o, lse, kbar, vbar)
    ctx.cfg = (block, scale, impl)
    ctx.mark_non_differentiable(lse, kbar, vbar)


def _attention_grad(ctx, dout, _dlse, _dkbar, _dvbar):
    q, k, v, o, lse, kbar, vbar = ctx.saved_tensors
    dq, dk, dv = _attention_bwd(q, k, v, o, lse, kbar, vbar, dout, *ctx.cfg)
    return dq, dk, dv, None, None, None


_attention_fwd.register_autograd(_attention_grad, setup_context=_attention_setup)


def _split_qkv(qkv, n_head):
    """The thirds of a packed (B, T, 3C) projection as (B, T, H, D) views."""
    B, T, C3 = qkv.shape
    C = C3 // 3
    return tuple(qkv[..., i * C:(i + 1) * C].view(B, T, n_head, C // n_head) for i in range(3))


@torch.library.custom_op("sqrtblock::attention_qkv_fwd", mutates_args=())
def _attention_qkv_fwd(qkv: torch.Tensor, n_head: int, block: Optional[int],
                       scale: Optional[float], impl: str
                       ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return sqrt_block_forward(*_split_qkv(qkv, n_head), block, scale, impl)


@_attention_qkv_fwd.register_fake
def _(qkv, n_head, block, scale, impl):
    B, T, C3 = qkv.shape
    H, D = n_head, C3 // 3 // n_head
    _, _, Gc = _fake_geometry(T, block)
    return (qkv.new_empty((B, T, H, D)), qkv.new_empty((B, H, T), dtype=torch.float32),
            qkv.new_empty((B, H, Gc, D)), qkv.new_empty((B, H, Gc, D)))


@torch.library.custom_op("sqrtblock::attention_qkv_bwd", mutates_args=())
def _attention_qkv_bwd(qkv: torch.Tensor, o: torch.Tensor, lse: torch.Tensor,
                       kbar: torch.Tensor, vbar: torch.Tensor, dout: torch.Tensor, n_head: int,
                       block: Optional[int], scale: Optional[float], impl: str) -> torch.Tensor:
    """dQ, dK, dV written straight into the thirds of one packed (B, T, 3C) gradient."""
    dqkv = torch.empty(qkv.shape, dtype=qkv.dtype, device=qkv.device)
    sqrt_block_backward(*_split_qkv(qkv, n_head), o, lse, kbar, vbar, dout, block, scale, impl,
                        out=_split_qkv(dqkv, n_head))
    return dqkv


@_attention_qkv_bwd.register_fake
def _(qkv, o, lse, kbar, vbar, dout, n_head, block, scale, impl):
    return qkv.new_empty(qkv.shape)


def _attention_qkv_setup(ctx, inputs, output):
    qkv, n_head, block, scale, impl = inputs
    o, lse, kbar, vbar = output
    ctx.save_for_backward(qkv, o, lse, kbar, vbar)
    ctx.cfg = (n_head, block, scale, impl)
    ctx.mark_non_differentiable(lse, kbar, vbar)


def _attention_qkv_grad(ctx, dout, _dlse, _dkbar, _dvbar):
    qkv, o, lse, kbar, vbar = ctx.saved_tensors
    return _attention_qkv_bwd(qkv, o, lse, kbar, vbar, dout, *ctx.cfg), None, None, None, None


_attention_qkv_fwd.register_autograd(_attention_qkv_grad, setup_context=_attention_qkv_setup)


def sqrt_block_attention_qkv(qkv, n_head, block=None, scale=None, impl="auto"):
    """``sqrt_block_attention`` on the thirds (Q, K, V) of one packed (B, T, 3C)
    projection, contiguous, C = n_head * D: the kernels read it in place, and the
    backward writes dQ, dK, dV into one (B, T, 3C) gradient, so the projection's
    backward is a single GEMM and needs no gradient adds (the
    ``sqrtblock::attention_qkv_fwd/bwd`` custom ops)."""
    if qkv.dim() != 3 or qkv.shape[-1] % (3 * n_head) != 0:
        raise ValueError(f"qkv must be (B, T, 3 * n_head * D), got {tuple(qkv.shape)}")
    return _attention_qkv_fwd(qkv.contiguous(), int(n_head), block, scale, impl)[0]


def sqrt_block_attention(q, k, v, block=None, scale=None, impl="auto"):
    """Differentiable sqrt-block attention on (B, T, H, D) CUDA views -> O (B, T, H, D).

    One ``sqrtblock::attention_fwd`` custom op (its backward is
    ``sqrtblock::attention_bwd``); LSE and the block summaries it also returns
    are saved for the backward and are not differentiable."""
    return _attention_fwd(q, k, v, block, scale, impl)[0]


# ---- reference-semantics mode ---------------------------------------------------

_refsem_workspaces: dict[tuple, torch.Tensor] = {}


def _refsem_workspace(device: torch.device, shape: tuple) -> torch.Tensor:
    """Scratch for one (B, T, H, D) reference-semantics problem (no initialisation needed)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx,) + tuple(int(x) for x in shape)
    with _ws_lock:
        ws = _refsem_workspaces.get(key)
        if ws is None:
            nbytes = int(_lib.lib().sqb_refsem_workspace_bytes(*shape))
            if nbytes == 0:
                raise ValueError(f"reference-semantics attention does not support (B, T, H, D) = "
                                 f"{tuple(shape)} (T must be a perfect square with sqrt(T) <= 64, "
                                 "D <= 128)")
            ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
            _refsem_workspaces[key] = ws
        return ws


def _refsem_check_T(T: int) -> int:
    L = math.isqrt(max(T, 0))
    if L * L != T or T <= 0:
        # the reference's block_geometry (model/custom_attention.py:75-77)
        raise ValueError(f"sequence length {T} must be a perfect square")
    return L


def reference_forward(q, k, v, scale=None):
    """Reference-semantics forward -> (o, glob, summary).

    The attention core of the reference's own sqrt_block module
    (model/custom_attention.py:183-227) on (B, T, H, D) CUDA views; T must be a
    perfect square.  o: (B, T, H, D); glob: (B, H, G, G) fp32; summary:
    (B, H, G, L) fp32 (both saved for the backward).
    """
    q, k, v = _prep(q, "q"), _prep(k, "k"), _prep(v, "v")
    if not (q.shape == k.shape == v.shape):
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in _DTYPES:
        raise TypeError(f"q, k, v must share a float32 or bfloat16 dtype, got "
                        f"{q.dtype}, {k.dtype}, {v.dtype}")
    B, T, H, D = q.shape
    L = _refsem_check_T(T)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = q.device
    o = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
    glob = torch.empty((B, H, L, L), dtype=torch.float32, device=dev)
    summary = torch.empty((B, H, L, L), dtype=torch.float32, device=dev)
    ws = _refsem_workspace(dev, (B, T, H, D))
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = _lib.strides_array(_strides(q), _strides(k), _strides(v), _strides(o))
    rc = _lib.lib().sqb_refsem_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                   glob.data_ptr(), summary.data_ptr(), B, T, H, D, st,
                                   _DTYPES[q.dtype], float(scale), ws.data_ptr(), ws.numel(),
                                   stream)
    _lib.check("sqb_refsem_fwd", rc)
    return o, glob, summary


def reference_backward(q, k, v, glob, summary, dout, scale=None):
    """Reference-semantics backward -> (dq, dk, dv), each (B, T, H, D)."""
    q, k, v, dout = _prep(q, "q"), _prep(k, "k"), _prep(v, "v"), _prep(dout, "dout")
    if dout.dtype != q.dtype:
        dout = dout.to(q.dtype)
    B, T, H, D = q.shape
    _refsem_check_T(T)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = q.device
    dq = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
    dk = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
    dv = torch.empty((B, T, H, D), dtype=q.dtype, device=dev)
    ws = _refsem_workspace(dev, (B, T, H, D))
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = _lib.strides_array(*(_strides(t) for t in (q, k, v, dout, dq, dk, dv)))
    rc = _lib.lib().sqb_refsem_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), dout.data_ptr(),
                                   glob.contiguous().data_ptr(), summary.contiguous().data_ptr(),
                                   dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, T, H, D, st,
                                   _DTYPES[q.dtype], float(scale), ws.data_ptr(), ws.numel(),
                                   stream)
    _lib.check("sqb_refsem_bwd", rc)
    return dq, dk, dv


@torch.library.custom_op("sqrtblock::reference_fwd", mutates_args=())
def _reference_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float]
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return reference_forward(q, k, v, scale)


@_reference_fwd.register_fake
def _(q, k, v, scale):
    B, T, H, D = q.shape
    L = _refsem_check_T(int(T))
    return (q.new_empty((B, T, H, D)), q.new_empty((B, H, L, L), dtype=torch.float32),
            q.new_empty((B, H, L, L), dtype=torch.float32))


@torch.library.custom_op("sqrtblock::reference_bwd", mutates_args=())
def _reference_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, glob: torch.Tensor,
                   summary: torch.Tensor, dout: torch.Tensor, scale: Optional[float]
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return reference_backward(q, k, v, glob, summary, dout, scale)


@_reference_bwd.register_fake
def _(q, k, v, glob, summary, dout, scale):
    return tuple(q.new_empty(q.shape) for _ in range(3))


def _reference_setup(ctx, inputs, output):
    q, k, v, scale = inputs
    o, glob, summary = output
    ctx.save_for_backward(q, k, v, glob, summary)
    ctx.scale = scale
    ctx.mark_non_differentiable(glob, summary)


def _reference_grad(ctx, dout, _dglob, _dsummary):
    q, k, v, glob, summary = ctx.saved_tensors
    dq, dk, dv = _reference_bwd(q, k, v, glob, summary, dout, ctx.scale)
    return dq, dk, dv, None


_reference_fwd.register_autograd(_reference_grad, setup_context=_reference_setup)


def reference_attention(q, k, v, scale=None):
    """Differentiable reference-semantics attention on (B, T, H, D) CUDA views -> O
    (the ``sqrtblock::reference_fwd`` custom op)."""
    return _reference_fwd(q, k, v, scale)[0]


# ---- training caller: fused token cross-entropy (include/sqb_train.h) ------------


@torch.library.custom_op("sqrtblock::xent_fwd", mutates_args=())
def _xent_fwd(x: torch.Tensor, t: torch.Tensor
              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rows x (N, V) (row pitch x.stride(0)), targets t (N,) int64 ->
    (mean loss over counted rows, per-row log-sum-exp, counted rows)."""
    N, V = x.shape
    loss = torch.empty(N, dtype=torch.float32, device=x.device)
    lse = torch.empty(N, dtype=torch.float32, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.check("sqb_xent_fwd", _lib.lib().sqb_xent_fwd(
        x.data_ptr(), t.data_ptr(), loss.data_ptr(), lse.data_ptr(), N, V, x.stride(0),
        _DTYPES[x.dtype], stream))
    counted = (t >= 0).sum().to(torch.float32)
    return loss.sum() / counted, lse, counted


@_xent_fwd.register_fake
def _(x, t):
    f32 = torch.float32
    return x.new_empty((), dtype=f32), x.new_empty((x.shape[0],), dtype=f32), \
        x.new_empty((), dtype=f32)


@torch.library.custom_op("sqrtblock::xent_bwd", mutates_args=())
def _xent_bwd(x: torch.Tensor, t: torch.Tensor, lse: torch.Tensor, scale: torch.Tensor
              ) -> torch.Tensor:
    """Gradient rows (N, x.stride(0)) in x's dtype: scale * (softmax - onehot) in
    the first V columns (zeros past V)."""
    N, V = x.shape
    ld = x.stride(0)
    dbuf = torch.empty(N, ld, dtype=x.dtype, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.check("sqb_xent_bwd", _lib.lib().sqb_xent_bwd(
        x.data_ptr(), t.data_ptr(), lse.data_ptr(), scale.data_ptr(), dbuf.data_ptr(), N, V,
        ld, _DTYPES[x.dtype], stream))
    return dbuf


@_xent_bwd.register_fake
def _(x, t, lse, scale):
    return x.new_empty((x.shape[0], x.stride(0)))


def _xent_setup(ctx, inputs, output):
    x, t = inputs
    _, lse, counted = output
    ctx.save_for_backward(x, t, lse, counted)
    ctx.mark_non_differentiable(lse, counted)


def _xent_grad(ctx, grad, _dlse, _dcounted):
    x, t, lse, counted = ctx.saved_tensors
    scale = (grad.to(torch.float32) / counted).reshape(1).contiguous()
    return _xent_bwd(x, t, lse, scale)[:, :x.shape[1]], None


_xent_fwd.register_autograd(_xent_grad, setup_context=_xent_setup)


def cross_entropy(logits, targets):
    """Mean next-token cross-entropy of CUDA logits (..., V) against integer targets
    (negative = ignored), as ``F.cross_entropy`` computes it (fp32 math, mean over
    the counted tokens), fused: the logits are read once forward and the gradient
    written once backward, in the logits' dtype (``sqrtblock::xent_fwd/bwd``)."""
    V = logits.shape[-1]
    x = logits.reshape(-1, V)
    if x.stride(-1) != 1 or x.stride(0) < V:
        x = x.contiguous()
    t = targets.reshape(-1).to(torch.int64).contiguous()
    if x.dtype not in _DTYPES or not x.is_cuda or t.numel() != x.shape[0]:
        raise ValueError("cross_entropy: CUDA float32/bfloat16 logits (..., V) and one "
                         "target per row")
    return _xent_fwd(x, t)[0]


# ---- training caller: fused LayerNorm (include/sqb_train.h) -----------------------


def layer_norm_supported(x, weight) -> bool:
    """The library's LayerNorm takes CUDA fp32 rows of C = 128k <= 1024 with an fp32
    weight (the GPT caller's residual stream); other inputs use ``F.layer_norm``."""
    C = x.shape[-1]
    return (x.is_cuda and x.dtype == torch.float32 and weight is not None
            and weight.dtype == torch.float32 and C % 128 == 0 and C <= 1024)


@torch.library.custom_op("sqrtblock::layernorm_fwd", mutates_args=())
def _layernorm_fwd(x2: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], eps: float,
                   out_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rows x2 (N, C) fp32 contiguous -> (y (N, C) in out_dtype, mean, rstd)."""
    N, C = x2.shape
    y = torch.empty((N, C), dtype=out_dtype, device=x2.device)
    mean = torch.empty(N, dtype=torch.float32, device=x2.device)
    rstd = torch.empty(N, dtype=torch.float32, device=x2.device)
    stream = torch.cuda.current_stream(x2.device).cuda_stream
    _lib.check("sqb_layernorm_fwd", _lib.lib().sqb_layernorm_fwd(
        x2.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None, y.data_ptr(),
        _DTYPES[out_dtype], mean.data_ptr(), rstd.data_ptr(), N, C, float(eps), stream))
    return y, mean, rstd


@_layernorm_fwd.register_fake
def _(x2, w, b, eps, out_dtype):
    N, C = x2.shape
    f32 = torch.float32
    return (x2.new_empty((N, C), dtype=out_dtype), x2.new_empty((N,), dtype=f32),
            x2.new_empty((N,), dtype=f32))


@torch.library.custom_op("sqrtblock::layernorm_bwd", mutates_args=())
def _layernorm_bwd(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor, mean: torch.Tensor,
                   rstd: torch.Tensor, has_bias: bool
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dx (N, C) fp32, dw (C,), db (C,), or an empty db without a bias)."""
    N, C = x2.shape
    dx = torch.empty((N, C), dtype=torch.float32, device=x2.device)
    dw = torch.empty(C, dtype=torch.float32, device=x2.device)
    db = torch.empty(C if has_bias else 0, dtype=torch.float32, device=x2.device)
    wsb = _lib.lib().sqb_layernorm_workspace_bytes(N, C)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=x2.device)
    stream = torch.cuda.current_stream(x2.device).cuda_stream
    _lib.check("sqb_layernorm_bwd", _lib.lib().sqb_layernorm_bwd(
        dy2.data_ptr(), _DTYPES[dy2.dtype], x2.data_ptr(), w.data_ptr(), mean.data_ptr(),
        rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr() if has_bias else None,
        ws.data_ptr(), wsb, N, C, stream))
    return dx, dw, db


@_layernorm_bwd.register_fake
def _(dy2, x2, w, mean, rstd, has_bias):
    N, C = x2.shape
    f32 = torch.float32
    return (x2.new_empty((N, C), dtype=f32), x2.new_empty((C,), dtype=f32),
            x2.new_empty((C if has_bias else 0,), dtype=f32))


def _layernorm_setup(ctx, inputs, output):
    x2, w, b, eps, out_dtype = inputs
    _, mean, rstd = output
    ctx.save_for_backward(x2, w, mean, rstd)
    ctx.has_bias = b is not None
    ctx.mark_non_differentiable(mean, rstd)


def _layernorm_grad(ctx, dy, _dmean, _drstd):
    x2, w, mean, rstd = ctx.saved_tensors
    N, C = x2.shape
    dy2 = dy.reshape(N, C)
    if dy2.dtype not in _DTYPES:
        dy2 = dy2.float()
    dx, dw, db = _layernorm_bwd(dy2.contiguous(), x2, w, mean, rstd, ctx.has_bias)
    return dx, dw, (db if ctx.has_bias else None), None, None


_layernorm_fwd.register_autograd(_layernorm_grad, setup_context=_layernorm_setup)


@torch.library.custom_op("sqrtblock::add_layernorm_fwd", mutates_args=())
def _add_layernorm_fwd(x2: torch.Tensor, h2: torch.Tensor, w: torch.Tensor,
                       b: Optional[torch.Tensor], eps: float, out_dtype: torch.dtype
                       ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rows x2 (N, C) fp32 and h2 (N, C) fp32/bf16 -> (x2 + h2 fp32, its LayerNorm in
    out_dtype, mean, rstd)."""
    N, C = x2.shape
    xo = torch.empty((N, C), dtype=torch.float32, device=x2.device)
    y = torch.empty((N, C), dtype=out_dtype, device=x2.device)
    mean = torch.empty(N, dtype=torch.float32, device=x2.device)
    rstd = torch.empty(N, dtype=torch.float32, device=x2.device)
    stream = torch.cuda.current_stream(x2.device).cuda_stream
    _lib.check("sqb_add_layernorm_fwd", _lib.lib().sqb_add_layernorm_fwd(
        x2.data_ptr(), h2.data_ptr(), _DTYPES[h2.dtype], xo.data_ptr(), w.data_ptr(),
        b.data_ptr() if b is not None else None, y.data_ptr(), _DTYPES[out_dtype],
        mean.data_ptr(), rstd.data_ptr(), N, C, float(eps), stream))
    return xo, y, mean, rstd


@_add_layernorm_fwd.register_fake
def _(x2, h2, w, b, eps, out_dtype):
    N, C = x2.shape
    f32 = torch.float32
    return (x2.new_empty((N, C), dtype=f32), x2.new_empty((N, C), dtype=out_dtype),
            x2.new_empty((N,), dtype=f32), x2.new_empty((N,), dtype=f32))


@torch.library.custom_op("sqrtblock::add_layernorm_bwd", mutates_args=())
def _add_layernorm_bwd(dy2: torch.Tensor, xo2: torch.Tensor, w: torch.Tensor,
                       mean: torch.Tensor, rstd: torch.Tensor, dres: Optional[torch.Tensor],
                       has_bias: bool, h_bf16: bool
                       ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dx fp32 = the gradient of x and h, dh as bf16 (empty unless h_bf16), dw, db)."""
    N, C = xo2.shape
    dx = torch.empty((N, C), dtype=torch.float32, device=xo2.device)
    dh = torch.empty((N, C) if h_bf16 else (0,), dtype=torch.bfloat16, device=xo2.device)
    dw = torch.empty(C, dtype=torch.float32, device=xo2.device)
    db = torch.empty(C if has_bias else 0, dtype=torch.float32, device=xo2.device)
    wsb = _lib.lib().sqb_layernorm_workspace_bytes(N, C)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=xo2.device)
    stream = torch.cuda.current_stream(xo2.device).cuda_stream
    _lib.check("sqb_add_layernorm_bwd", _lib.lib().sqb_add_layernorm_bwd(
        dy2.data_ptr(), _DTYPES[dy2.dtype], xo2.data_ptr(), w.data_ptr(), mean.data_ptr(),
        rstd.data_ptr(), dres.data_ptr() if dres is not None else None, dx.data_ptr(),
        dh.data_ptr() if h_bf16 else None, dw.data_ptr(),
        db.data_ptr() if has_bias else None, ws.data_ptr(), wsb, N, C, stream))
    return dx, dh, dw, db


@_add_layernorm_bwd.register_fake
def _(dy2, xo2, w, mean, rstd, dres, has_bias, h_bf16):
    N, C = xo2.shape
    f32 = torch.float32
    return (xo2.new_empty((N, C), dtype=f32),
            xo2.new_empty((N, C) if h_bf16 else (0,), dtype=torch.bfloat16),
            xo2.new_empty((C,), dtype=f32), xo2.new_empty((C if has_bias else 0,), dtype=f32))


def _add_layernorm_setup(ctx, inputs, output):
    x2, h2, w, b, eps, out_dtype = inputs
    xo, _, mean, rstd = output
    ctx.save_for_backward(xo, w, mean, rstd)
    ctx.has_bias = b is not None
    ctx.h_dtype = h2.dtype
    ctx.mark_non_differentiable(mean, rstd)


def _add_layernorm_grad(ctx, dxo, dy, _dmean, _drstd):
    xo, w, mean, rstd = ctx.saved_tensors
    N, C = xo.shape
    if dy is None:
        dy = torch.zeros((N, C), dtype=torch.float32, device=xo.device)
    dy2 = dy.reshape(N, C)
    if dy2.dtype not in _DTYPES:
        dy2 = dy2.float()
    dres = dxo.reshape(N, C).float().contiguous() if dxo is not None else None
    h_bf16 = ctx.h_dtype == torch.bfloat16
    dx, dh, dw, db = _add_layernorm_bwd(dy2.contiguous(), xo, w, mean, rstd, dres,
                                        ctx.has_bias, h_bf16)
    dh_out = dh if h_bf16 else dx.to(ctx.h_dtype, copy=True)
    return dx, dh_out, dw, (db if ctx.has_bias else None), None, None


_add_layernorm_fwd.register_autograd(_add_layernorm_grad, setup_context=_add_layernorm_setup)


def add_layer_norm(x, h, weight, bias=None, eps=1e-5, out_dtype=torch.float32):
    """(x + h, LayerNorm(x + h)) for CUDA fp32 ``x`` and fp32 or bf16 ``h`` of the same
    shape (``layer_norm_supported(x, weight)``): the sum in fp32 as torch adds them,
    the LayerNorm as ``layer_norm``; one kernel each way (the
    ``sqrtblock::add_layernorm_fwd/bwd`` custom ops)."""
    C = x.shape[-1]
    x2 = x.reshape(-1, C).contiguous()
    h2 = h.reshape(-1, C).contiguous()
    b = bias.contiguous() if bias is not None else None
    xo, y, _, _ = _add_layernorm_fwd(x2, h2, weight.contiguous(), b, float(eps), out_dtype)
    return xo.view(x.shape), y.view(x.shape)


def add_layer_norm_supported(x, h, weight) -> bool:
    return (layer_norm_supported(x, weight) and h.shape == x.shape and h.is_cuda
            and h.dtype in (torch.float32, torch.bfloat16))


def layer_norm(x, weight, bias=None, eps=1e-5, out_dtype=torch.float32):
    """LayerNorm over the last dimension of CUDA fp32 ``x`` (see
    ``layer_norm_supported``), fp32 math; the output in ``out_dtype`` (fp32, or
    bf16 for a bf16 autocast consumer, which would cast it to that anyway).
    The ``sqrtblock::layernorm_fwd/bwd`` custom ops."""
    C = x.shape[-1]
    x2 = x.reshape(-1, C).contiguous()
    b = bias.contiguous() if bias is not None else None
    return _layernorm_fwd(x2, weight.contiguous(), b, float(eps), out_dtype)[0].view(x.shape)
