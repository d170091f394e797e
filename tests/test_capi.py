"""The C ABI library on CPU: it loads, exports every symbol include/sqrtblock.h
declares, and validates arguments without touching a device."""

import ctypes
import os
import re

import pytest

from llm_training_b200 import _lib
from oracle import sqrtblock_oracle as orc

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "sqrtblock.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sqb_[a-z_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 7
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES)


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.sqb_version() >= 100
    for code in range(0, 10):
        assert lib.sqb_strerror(code)
    assert b"unknown" in lib.sqb_strerror(12345)


@pytest.mark.parametrize("T", [1, 2, 15, 16, 17, 255, 256, 257, 1000, 1024, 4096, 8192, 16384,
                               32768, 65536, 100000])
def test_geometry_matches_oracle(T):
    assert _lib.geometry(T) == orc.geometry(T)
    assert _lib.geometry(T, 48) == orc.geometry(T, 48)


def test_workspace_bytes():
    assert _lib.workspace_bytes(1, 16384, 16, 128, 128) > 2 * 16 * 128 * 128 * 4
    assert _lib.workspace_bytes(0, 16, 1, 8, 16) == 0


def _fwd(**over):
    args = dict(q=1, k=1, v=1, o=1, lse=1, kbar=1, vbar=1, B=1, T=64, H=1, D=32, block=16,
                dtype=_lib.SQB_BF16, scale=0.1, impl=0, ws=1, wsb=1 << 30, stream=None)
    args.update(over)
    st = _lib.strides_array(*([(64 * 32, 32, 32)] * 4))
    a = args
    return _lib.lib().sqb_fwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["kbar"], a["vbar"],
                              a["B"], a["T"], a["H"], a["D"], a["block"], st, a["dtype"],
                              a["scale"], a["impl"], a["ws"], a["wsb"], a["stream"])


def test_fwd_argument_errors_need_no_device():
    assert _fwd(q=None) == 1           # SQB_ERR_ARG
    assert _fwd(T=0) == 1
    assert _fwd(block=0) == 1
    assert _fwd(dtype=7) == 2          # SQB_ERR_DTYPE
    assert _fwd(ws=None) == 5          # SQB_ERR_WORKSPACE
    assert _fwd(wsb=16) == 5
    assert _fwd(scale=0.0) == 1
    assert _fwd(kbar=None) == 1        # T=64, b=16 has summaries


def test_check_raises_with_message():
    with pytest.raises(_lib.SqrtBlockError, match="workspace"):
        _lib.check("sqb_fwd", 5)


def test_status_entry_points_reject_a_missing_workspace():
    lib = _lib.lib()
    assert lib.sqb_read_status(None, None, None) == 1      # SQB_ERR_ARG
    assert lib.sqb_attach_status(None, None, 0, None) == 1
