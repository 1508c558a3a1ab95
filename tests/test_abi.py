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
