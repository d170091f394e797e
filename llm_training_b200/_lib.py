"""ctypes binding of the C ABI in include/sqrtblock.h (libsqrtblock.so).

The shared library is built in-tree by ``python -m llm_training_b200.build``.
There is no fallback: if the library is missing or fails to load, ``lib()``
raises, and every op that needs it fails with that error.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIBPATH

SQB_F32 = 0
SQB_BF16 = 1

IMPL_AUTO = 0
IMPL_SIMT = 1
IMPL_TCGEN05 = 2
IMPLS = {"auto": IMPL_AUTO, "simt": IMPL_SIMT, "tcgen05": IMPL_TCGEN05}

SQB_OK = 0
SQB_ERR_TIMEOUT = 7

# Every symbol declared in include/sqrtblock.h, with its ctypes signature.
_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
SIGNATURES = {
    "sqb_version": (ctypes.c_int, []),
    "sqb_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "sqb_geometry": (ctypes.c_int, [_c_i64, _c_i64, ctypes.POINTER(_c_i64),
                                    ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64)]),
    "sqb_workspace_bytes": (ctypes.c_size_t, [_c_i64] * 5),
    "sqb_fwd": (ctypes.c_int, [_vp] * 7 + [_c_i64] * 5 + [ctypes.POINTER(_c_i64), ctypes.c_int,
                                                           ctypes.c_float, ctypes.c_int, _vp,
                                                           ctypes.c_size_t, _vp]),
    "sqb_bwd": (ctypes.c_int, [_vp] * 11 + [_c_i64] * 5 + [ctypes.POINTER(_c_i64), ctypes.c_int,
                                                            ctypes.c_float, ctypes.c_int, _vp,
                                                            ctypes.c_size_t, _vp]),
    "sqb_read_status": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(_c_i64)]),
    "sqb_read_status_noalloc": (ctypes.c_int, [_vp, ctypes.POINTER(_c_i64)]),
    "sqb_attach_status": (ctypes.c_int, [_vp, _vp, ctypes.c_uint32, _vp]),
    "sqb_bwd_noalloc": (ctypes.c_int, [_vp] * 11 + [_c_i64] * 5 + [ctypes.POINTER(_c_i64),
                                                                    ctypes.c_int, ctypes.c_float,
                                                                    ctypes.c_int, _vp]),
    "sqb_refsem_workspace_bytes": (ctypes.c_size_t, [_c_i64] * 4),
    "sqb_refsem_fwd": (ctypes.c_int, [_vp] * 6 + [_c_i64] * 4 + [ctypes.POINTER(_c_i64),
                                                                 ctypes.c_int, ctypes.c_float,
                                                                 _vp, ctypes.c_size_t, _vp]),
    "sqb_refsem_bwd": (ctypes.c_int, [_vp] * 9 + [_c_i64] * 4 + [ctypes.POINTER(_c_i64),
                                                                 ctypes.c_int, ctypes.c_float,
                                                                 _vp, ctypes.c_size_t, _vp]),
}

_lock = threading.Lock()
_lib = None


class SqrtBlockError(RuntimeError):
    """An sqb_* call returned an error code."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with code {code}: {msg}")
        self.code = code


# Training-caller helpers (include/sqb_train.h), bound on the same library.
TRAIN_SIGNATURES = {
    "sqb_xent_fwd": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                    ctypes.c_void_p]),
    "sqb_xent_bwd": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, _c_i64, _c_i64, _c_i64,
                                    ctypes.c_int, ctypes.c_void_p]),
    "sqb_layernorm_fwd": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int] +
                          [ctypes.c_void_p] * 2 + [_c_i64, _c_i64, ctypes.c_float,
                                                   ctypes.c_void_p]),
    "sqb_layernorm_workspace_bytes": (ctypes.c_size_t, [_c_i64, _c_i64]),
    "sqb_layernorm_bwd": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 8 +
                          [ctypes.c_size_t, _c_i64, _c_i64, ctypes.c_void_p]),
    "sqb_add_layernorm_fwd": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int] +
                              [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 2 +
                              [_c_i64, _c_i64, ctypes.c_float, ctypes.c_void_p]),
    "sqb_add_layernorm_bwd": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int] +
                              [ctypes.c_void_p] * 10 +
                              [ctypes.c_size_t, _c_i64, _c_i64, ctypes.c_void_p]),
}


def library_path() -> str:
    return os.environ.get("SQB_LIBRARY", LIBPATH)


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"sqrt-block CUDA library not found at {path}; build it with "
                    "`python -m llm_training_b200.build` (there is no CPU fallback)")
            handle = ctypes.CDLL(path)
            for name, (res, args) in {**SIGNATURES, **TRAIN_SIGNATURES}.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(fn: str, code: int) -> None:
    if code != SQB_OK:
        raise SqrtBlockError(fn, code, lib().sqb_strerror(code).decode())


def geometry(T: int, block: int | None = None):
    """(b, G, Gc) as the library computes it."""
    b, g, gc = _c_i64(), _c_i64(), _c_i64()
    check("sqb_geometry", lib().sqb_geometry(T, block or 0, ctypes.byref(b), ctypes.byref(g),
                                             ctypes.byref(gc)))
    return b.value, g.value, gc.value


def workspace_bytes(B, T, H, D, block) -> int:
    return int(lib().sqb_workspace_bytes(B, T, H, D, block))


def strides_array(*strides) -> ctypes.Array:
    flat = [int(s) for st in strides for s in st]
    return (_c_i64 * len(flat))(*flat)
