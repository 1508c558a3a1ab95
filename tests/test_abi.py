"""CPU: the C-ABI library loads, exports every declared symbol, and rejects bad
arguments on the host without touching a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT


def declared_functions():
    header = (ROOT / "include" / "ttn.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    names = set(re.findall(r"\b(ttn_[a-z0-9_]+)\s*\(", header))
    return sorted(names)


def test_header_and_binding_agree():
    from thintnpu_b200 import _lib
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    from thintnpu_b200 import _lib
    lib = _lib.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.library_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ttn_\w+)", out))
    assert set(declared_functions()) <= exported


def test_library_is_built_for_sm100a():
    from thintnpu_b200 import _lib
    out = subprocess.run(["cuobjdump", "--list-elf", str(_lib.library_path())],
                         capture_output=True, text=True)
    if out.returncode:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_status_strings_and_version():
    from thintnpu_b200 import _lib
    lib = _lib.lib()
    assert lib.ttn_version() >= 100
    assert lib.ttn_status_string(0) == b"TTN_OK"
    assert lib.ttn_status_string(2) == b"TTN_UNSUPPORTED"


def test_host_side_argument_errors_need_no_gpu():
    from thintnpu_b200 import _lib
    lib = _lib.lib()
    # unknown op code is rejected before any CUDA call
    d = _lib.TtnTensor()
    assert lib.ttn_binary(9, 1.0, ctypes.byref(d), ctypes.byref(d), ctypes.byref(d), None) == 1
    assert b"unknown op" in lib.ttn_last_error()
    # null descriptors
    assert lib.ttn_silu(None, None, None) == 1
    # even kernel size
    assert lib.ttn_maxpool(1, 0, 4, None, None, 1, 1, 1, 1, None) == 1
    assert b"odd" in lib.ttn_last_error()
    # bad flags in selection
    bad = _lib.TtnTensor()
    bad.ndim = 3
    bad.dtype = 0
    bad.sizes[0], bad.sizes[1], bad.sizes[2] = 1, 4, 9
    bad.strides[0], bad.strides[1], bad.strides[2] = 36, 9, 1
    bad.data = 16
    assert lib.ttn_select_f16(ctypes.byref(bad), 2, 64, None, 0, None, None, None) == 1
    # dfl decode rejects a non-positive stride before launching
    h = (ctypes.c_int64 * 1)(2)
    w = (ctypes.c_int64 * 1)(2)
    s = (ctypes.c_float * 1)(0.0)
    assert lib.ttn_dfl_decode_f16(None, 0, 0, None, 0, 0, 1, 1, 1, h, w, s, 1, None, None) == 1


def test_workspace_size_is_positive_and_monotone():
    from thintnpu_b200 import _lib
    lib = _lib.lib()
    small = lib.ttn_select_workspace_size(1, 8400, 80, 300, 0)
    big = lib.ttn_select_workspace_size(8, 8400, 80, 300, 0)
    agnostic = lib.ttn_select_workspace_size(1, 8400, 80, 300, 1)
    assert 0 < agnostic <= small < big
    assert small % 256 == 0
    assert lib.ttn_select_workspace_size(1, 8400, 80, 0, 0) >= 8400 * 4


def test_conv_and_depthwise_argument_errors_need_no_gpu():
    """The conv entry points check flags, shapes, alignment and the residual's form
    before any CUDA call (fake, aligned device addresses are never dereferenced)."""
    from thintnpu_b200 import _lib
    lib = _lib.lib()
    X, W, O, R = 1 << 20, 2 << 20, 3 << 20, 4 << 20  # 16-byte aligned fake addresses
    conv = lambda flags=1, co=64, k=3, s=1, x=X: lib.ttn_conv2d_nc1hwc0_f16(
        x, 1, 4, 8, 8, 4 * 8 * 8 * 16, W, None, co, k, s, flags, O, co * 64, None)
    assert conv(flags=8) == 1 and b"unknown flags" in lib.ttn_last_error()
    assert conv(k=5) == 2 and b"3x3" in lib.ttn_last_error()
    assert conv(co=40) == 2 and b"co % 16" in lib.ttn_last_error()
    assert conv(x=X + 2) == 1 and b"aligned" in lib.ttn_last_error()
    res = lambda flags=1, r=R, rbs=64 * 64: lib.ttn_conv2d_residual_nc1hwc0_f16(
        X, 1, 4, 8, 8, 4 * 8 * 8 * 16, W, None, 64, 3, 1, flags, r, rbs, O, 64 * 64, None)
    assert res(r=None) == 1 and b"null residual" in lib.ttn_last_error()
    assert res(flags=3) == 2 and b"NC1HWC0" in lib.ttn_last_error()
    assert res(r=R + 8) == 1 and b"residual" in lib.ttn_last_error()
    assert res(rbs=12) == 1 and b"residual" in lib.ttn_last_error()
    dw = lambda k=3, s=1, flags=1, x=X: lib.ttn_depthwise_nc1hwc0_f16(
        x, 1, 4, 8, 8, 4 * 8 * 8 * 16, W, None, k, s, flags, O, 4 * 8 * 8 * 16, None)
    assert dw(k=4) == 2 and b"odd kernel" in lib.ttn_last_error()
    assert dw(s=3) == 2
    assert dw(flags=2) == 1 and b"unknown flags" in lib.ttn_last_error()
    assert dw(x=X + 8) == 1 and b"aligned" in lib.ttn_last_error()
