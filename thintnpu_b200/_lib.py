"""ctypes binding of libttn.so, the C ABI declared in include/ttn.h.

Loading fails loudly: there is no CPU or PyTorch fallback for any op.  The
library is built in-tree by ``python -m thintnpu_b200.build`` (or
``__graft_entry__.build()``); set ``TTN_LIBRARY`` to load another copy.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

MAX_DIMS = 8
F16, F32 = 0, 1
SUB, MUL, DIV, ADD = 0, 1, 2, 3
NCHW, NC1HWC0 = 0, 1
SELECT_AGNOSTIC, SELECT_NAN_LAST, SELECT_SIGMOID = 1, 2, 4
ATTENTION_PRESCALE = 1
CONV_SILU, CONV_NCHW = 1, 2

STATUS = {0: "TTN_OK", 1: "TTN_INVALID_ARG", 2: "TTN_UNSUPPORTED", 3: "TTN_CUDA_ERROR",
          4: "TTN_TIMEOUT", 5: "TTN_DEVICE_FAULT_FLAG"}
UNSUPPORTED = 2

# Every symbol include/ttn.h declares (checked by the CPU test suite).
EXPORTS = (
    "ttn_version", "ttn_status_string", "ttn_last_error",
    "ttn_malloc", "ttn_free", "ttn_malloc_host", "ttn_free_host", "ttn_memcpy_async",
    "ttn_graph_create", "ttn_graph_begin", "ttn_graph_end", "ttn_graph_replay",
    "ttn_graph_close", "ttn_graph_destroy",
    "ttn_silu", "ttn_sigmoid", "ttn_binary", "ttn_binary_scalar", "ttn_add_silu_f16",
    "ttn_bias_silu_residual_nc1hwc0_f16",
    "ttn_copy", "ttn_cat", "ttn_nc1hwc0_to_nchw_f16", "ttn_nchw_to_nc1hwc0_f16",
    "ttn_upsample2x", "ttn_upsample2x_nc1hwc0_f16", "ttn_maxpool", "ttn_sppf_f16",
    "ttn_softmax", "ttn_dfl_decode_f16", "ttn_dfl_decode_trace_f16", "ttn_attention_f16", "ttn_attention_fault_f16",
    "ttn_conv2d_nc1hwc0_f16", "ttn_conv2d_residual_nc1hwc0_f16", "ttn_conv2d_pack_weights_f16",
    "ttn_conv2d_fault_f16", "ttn_conv2d_test_withhold_copies", "ttn_depthwise_nc1hwc0_f16",
    "ttn_select_workspace_size", "ttn_select_f16", "ttn_select_f16_static",
)


class TtnTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * MAX_DIMS), ("strides", ctypes.c_int64 * MAX_DIMS)]


class SelectTrace(ctypes.Structure):
    _fields_ = [("class_max", ctypes.c_void_p), ("stage1_indices", ctypes.c_void_p),
                ("gathered_scores", ctypes.c_void_p), ("top_values", ctypes.c_void_p),
                ("stage2_indices", ctypes.c_void_p), ("anchor_indices", ctypes.c_void_p),
                ("labels", ctypes.c_void_p)]


class TtnError(RuntimeError):
    """A libttn call returned a non-OK status."""

    def __init__(self, function: str, status: int, message: str):
        self.status = status
        super().__init__(f"{function}: {STATUS.get(status, status)}: {message}")


def library_path() -> Path:
    override = os.environ.get("TTN_LIBRARY")
    return Path(override) if override else Path(__file__).with_name("libttn.so")


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_TP = ctypes.POINTER(TtnTensor)

_SIGNATURES = {
    "ttn_version": (ctypes.c_int, []),
    "ttn_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ttn_last_error": (ctypes.c_char_p, []),
    "ttn_malloc": (ctypes.c_int, [ctypes.POINTER(_P), ctypes.c_size_t]),
    "ttn_free": (ctypes.c_int, [_P]),
    "ttn_malloc_host": (ctypes.c_int, [ctypes.POINTER(_P), ctypes.c_size_t]),
    "ttn_free_host": (ctypes.c_int, [_P]),
    "ttn_memcpy_async": (ctypes.c_int, [_P, _P, ctypes.c_size_t, ctypes.c_int, _P]),
    "ttn_graph_create": (ctypes.c_int, [ctypes.POINTER(_P)]),
    "ttn_graph_begin": (ctypes.c_int, [_P, _P]),
    "ttn_graph_end": (ctypes.c_int, [_P]),
    "ttn_graph_replay": (ctypes.c_int, [_P]),
    "ttn_graph_close": (ctypes.c_int, [_P]),
    "ttn_graph_destroy": (None, [_P]),
    "ttn_silu": (ctypes.c_int, [_TP, _TP, _P]),
    "ttn_sigmoid": (ctypes.c_int, [_TP, _TP, _P]),
    "ttn_binary": (ctypes.c_int, [ctypes.c_int, ctypes.c_float, _TP, _TP, _TP, _P]),
    "ttn_add_silu_f16": (ctypes.c_int, [_TP, _TP, _TP, _P]),
    "ttn_binary_scalar": (ctypes.c_int, [ctypes.c_int, ctypes.c_double, _TP, _TP, _P]),
    "ttn_bias_silu_residual_nc1hwc0_f16": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "ttn_copy": (ctypes.c_int, [_TP, _TP, _P]),
    "ttn_cat": (ctypes.c_int, [_I32, _TP, _I32, _TP, _P]),
    "ttn_nc1hwc0_to_nchw_f16": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P]),
    "ttn_nchw_to_nc1hwc0_f16": (ctypes.c_int, [_P, _I64, _I64, _I64, _P, _P]),
    "ttn_upsample2x": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "ttn_upsample2x_nc1hwc0_f16": (ctypes.c_int, [_P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "ttn_maxpool": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _I32, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "ttn_sppf_f16": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _I64, _I32, _P]),
    "ttn_softmax": (ctypes.c_int, [_TP, _I32, ctypes.c_float, _TP, _P]),
    "ttn_dfl_decode_f16": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I32,
                                          ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                                          ctypes.POINTER(ctypes.c_float), _I32, _P, _P]),
    "ttn_dfl_decode_trace_f16": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I32,
                                                ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                                                ctypes.POINTER(ctypes.c_float), _I32, _P, _P, _P]),
    "ttn_attention_f16": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, ctypes.POINTER(_I64),
                                         ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                                         ctypes.c_float, ctypes.c_uint32, _P]),
    "ttn_attention_fault_f16": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "ttn_conv2d_nc1hwc0_f16": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I32, _I32,
                                              ctypes.c_uint32, _P, _I64, _P]),
    "ttn_conv2d_residual_nc1hwc0_f16": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I32, _I32,
                                                       ctypes.c_uint32, _P, _I64, _P, _I64, _P]),
    "ttn_conv2d_pack_weights_f16": (ctypes.c_int, [_P, _I64, _I64, _I32, _P, _P]),
    "ttn_conv2d_fault_f16": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "ttn_conv2d_test_withhold_copies": (None, []),
    "ttn_depthwise_nc1hwc0_f16": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I32, _I32,
                                                 ctypes.c_uint32, _P, _I64, _P]),
    "ttn_select_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, ctypes.c_uint32]),
    "ttn_select_f16": (ctypes.c_int, [_TP, _I64, ctypes.c_uint32, _P, ctypes.c_size_t, _P,
                                      ctypes.POINTER(SelectTrace), _P]),
    "ttn_select_f16_static": (ctypes.c_int, [_TP, _I64, ctypes.c_uint32, _P,
                                             ctypes.POINTER(SelectTrace), _P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libttn.so once; raise ImportError with the reason when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise ImportError(f"libttn.so not found at {path}; build it with "
                          "`python -m thintnpu_b200.build` (no fallback implementation exists)")
    handle = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = handle
    return handle


def check(function: str, status: int) -> None:
    if status:
        message = lib().ttn_last_error().decode(errors="replace")
        raise TtnError(function, status, message)


def call(function: str, *args) -> None:
    """Call a status-returning entry point and raise TtnError on failure."""
    check(function, getattr(lib(), function)(*args))
