"""CPU-side checks of the C ABI: the library loads, exports every entry point include/redline_b200.h declares,
and rejects bad arguments with a status and a message before touching a device (no kernel is launched here)."""

import ctypes
import os
import re

import pytest

from redline_tiny_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "redline_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rl_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from redline_tiny_b200 import build
    build.build()
    return L.lib()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"


def test_argument_errors_are_reported_without_a_device(lib):
    st = lib.rl_quantize_bfp16(None, 0, 8, 8, 0, None, None, None)
    assert st == L.RL_ERR_ARGUMENT
    assert b"NULL" in lib.rl_last_error()
    buf = ctypes.create_string_buffer(64)
    st = lib.rl_quantize_bfp16(buf, 0, 8, 12, 0, None, None, None)
    assert st == L.RL_ERR_ARGUMENT and b"K % 8" in lib.rl_last_error()
    st = lib.rl_linear_bfp16(buf, 128, 100, buf, 256, None, 0, buf, 1, None)
    assert st == L.RL_ERR_ARGUMENT
    st = lib.rl_linear_bfp16(buf, 128, 128, buf, 256, None, 1, buf, 1, None)   # bias epilogue without bias
    assert st == L.RL_ERR_ARGUMENT and b"bias" in lib.rl_last_error()
    st = lib.rl_pack_b(buf, 0, 64, 100, buf, None)
    assert st == L.RL_ERR_ARGUMENT


def test_misaligned_pointer_rejected(lib):
    buf = ctypes.create_string_buffer(256)
    p = ctypes.addressof(buf)
    p = (p + 15) // 16 * 16 + 2
    st = lib.rl_quantize_bfp16(p, 1, 8, 8, 0, None, None, None)
    assert st == L.RL_ERR_ALIGNMENT


def test_python_wrapper_raises(lib):
    with pytest.raises(L.RedlineError) as e:
        L.call("rl_pack_b", None, 0, 64, 128, None, None)
    assert e.value.status == L.RL_ERR_ARGUMENT
