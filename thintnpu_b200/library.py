"""``torch.ops`` registrations that mirror the reference's operator schemas on CUDA.

Namespaces and schemas follow the reference (backend.cpp:321-356,
flow_ops.cpp:255-266, selection_flow.cpp:503-514, conv_blocked.cpp:199-206):

* ``thin_backend::{add, sigmoid, maxpool2d, upsample_nearest2d}``
* ``thin_native_flow::{maxpool, upsample, detection_select, detection_select_trace}``,
  the convolutions ``conv`` (conv_flow.cpp:630-646), ``depthwise``
  (depthwise_flow.cpp:225-233) and ``pack_input``, plus the fused ops of this
  build: ``silu_``, ``sppf``, ``softmax``, ``dfl_decode``, ``bias_silu_residual``
* ``thin_blocked::{pack, unpack, conv}`` (conv_blocked.cpp:198-210)

Each op has a CUDA kernel (libttn through ``thintnpu_b200.ops``), a Meta kernel
for shape inference, and an Autograd fallthrough (the ops are inference-only and
check ``requires_grad`` themselves, as the reference does).  Registration runs
once, on import.
"""
from __future__ import annotations

from typing import List

import torch
from torch.library import Library

from . import ops

_LIBS: List[Library] = []


def _lib(namespace: str) -> Library:
    lib = Library(namespace, "DEF")
    _LIBS.append(lib)
    return lib


def _register(lib: Library, schema: str, cuda, meta) -> None:
    name = schema.split("(", 1)[0]
    lib.define(schema)
    lib.impl(name, cuda, "CUDA")
    lib.impl(name, meta, "Meta")
    lib.impl(name, torch.library.fallthrough_kernel, "AutogradCUDA")
    lib.impl(name, torch.library.fallthrough_kernel, "AutogradMeta")


def _require(cond: bool, message: str) -> None:
    if not cond:
        raise RuntimeError(message)


# --------------------------------------------------------------- thin_backend

def _add_cuda(x, y):
    _require(x.device == y.device, "add requires tensors on the same device")
    _require(x.dtype == y.dtype and x.shape == y.shape and x.dtype in (torch.float32, torch.float16),
             "add requires matching float32/float16 tensors")
    return ops.add(x, y)


def _add_meta(x, y):
    _require(x.shape == y.shape and x.dtype == y.dtype and x.dtype in (torch.float32, torch.float16),
             "add requires matching float32/float16 tensors")
    return torch.empty_like(x)


def _sigmoid_meta(x):
    _require(x.dtype in (torch.float32, torch.float16), "sigmoid supports float32 and float16")
    return torch.empty_like(x)


def _maxpool2d_cuda(x):
    _require(x.dim() == 4 and x.size(1) > 0 and x.size(2) > 0 and x.size(3) > 0,
             "maxpool2d requires NCHW with positive C/H/W")
    return ops.maxpool2d(x, 5)


def _nchw_meta(x):
    _require(x.dim() == 4 and x.dtype in (torch.float32, torch.float16),
             "requires float32/float16 NCHW")
    return x


def _upsample_meta(x):
    _require(x.dim() == 4 and x.dtype in (torch.float32, torch.float16),
             "upsample_nearest2d supports float32/float16 NCHW")
    _require(x.size(1) > 0 and x.size(2) > 0 and x.size(3) > 0, "C, H, W must be positive")
    return x.new_empty((x.size(0), x.size(1), 2 * x.size(2), 2 * x.size(3)))


# ----------------------------------------------------------- thin_native_flow

def _blocked_meta(x):
    _require(x.dim() == 5 and x.size(4) == 16 and x.dtype == torch.float16,
             "expected aligned contiguous FP16 NC1HWC0 input, C0=16")


def _maxpool_meta(x, kernel):
    _blocked_meta(x)
    _require(kernel >= 1 and kernel % 2 == 1, "maxpool kernel must be a positive odd integer")
    return torch.empty_like(x)


def _upsample_blocked_meta(x):
    _blocked_meta(x)
    n, c1, h, w, _ = x.shape
    return x.new_empty((n, c1, 2 * h, 2 * w, 16))


def _select_cuda(decoded, max_det, agnostic=False):
    return ops.detection_select(decoded, max_det, agnostic)


def _select_meta(decoded, max_det, agnostic=False):
    _require(decoded.dim() == 3 and decoded.dtype == torch.float16,
             "detection_select expects inference-only device FP16 [B,A,4+nc]")
    _require(decoded.size(2) > 4 and max_det >= 0, "detection_select requires nc > 0 and max_det >= 0")
    k = min(max_det, decoded.size(1))
    return decoded.new_empty((decoded.size(0), k, 6), dtype=torch.float32)


def _select_trace_cuda(decoded, max_det, agnostic=False):
    return ops.detection_select(decoded, max_det, agnostic, trace=True)


def _select_trace_meta(decoded, max_det, agnostic=False):
    out = _select_meta(decoded, max_det, agnostic)
    b, a, c = decoded.shape
    k, nc = out.size(1), c - 4
    new = decoded.new_empty
    return [out, new((b, a)), new((b, k), dtype=torch.int64), new((b, 0 if agnostic else k, nc)),
            new((b, k)), new((b, 0 if agnostic else k), dtype=torch.int64),
            new((b, k), dtype=torch.int64), new((b, k), dtype=torch.int64)]


def _silu__cuda(x):
    return ops.silu_(x)


def _silu__meta(x):
    return x


def _sppf_meta(x, kernel=5):
    _blocked_meta(x)
    n, c1, h, w, _ = x.shape
    return x.new_empty((n, 4 * c1, h, w, 16))


def _softmax_cuda(x, dim, scale=1.0, half_to_float=False):
    return ops.softmax(x, dim, half_to_float=half_to_float, scale=scale)


def _softmax_meta(x, dim, scale=1.0, half_to_float=False):
    return x.new_empty(x.shape, dtype=torch.float32 if half_to_float else x.dtype)


def _decode_cuda(box, cls, heights, widths, strides, xywh=True):
    return ops.dfl_decode(box, cls, list(zip(heights, widths)), strides, xywh)


def _decode_meta(box, cls, heights, widths, strides, xywh=True):
    return box.new_empty((box.size(0), 4 + cls.size(1), box.size(2)))


def _bsr_cuda(x, bias, residual):
    return ops.bias_silu_residual(x, bias, residual)


def _bsr_meta(x, bias, residual):
    return torch.empty_like(x)


def _conv_out_shape(x, co, kernel, stride, nchw):
    n, _, h, w, _ = x.shape
    pad = (kernel - 1) // 2
    oh, ow = (h + 2 * pad - kernel) // stride + 1, (w + 2 * pad - kernel) // stride + 1
    return (n, co, oh, ow) if nchw else (n, co // 16, oh, ow, 16)


def _conv_cuda(x, packed, bias, co, kernel, stride, fused=True, nchw_output=False):
    return ops.conv2d(x, packed, bias, co, kernel, stride, silu=fused, nchw=nchw_output)


def _conv_meta(x, packed, bias, co, kernel, stride, fused=True, nchw_output=False):
    _blocked_meta(x)
    _require((kernel == 1 and stride == 1) or (kernel in (3, 6) and stride in (1, 2)),
             "expected point stride1 or spatial stride1/2")
    _require(co > 0 and (nchw_output or co % 16 == 0), "blocked outputs require aligned channels")
    return x.new_empty(_conv_out_shape(x, co, kernel, stride, nchw_output))


def _depthwise_cuda(x, packed, bias, kernel, stride, fused=True):
    return ops.depthwise(x, packed, bias, kernel, stride, silu=fused)


def _depthwise_meta(x, packed, bias, kernel, stride, fused=True):
    _blocked_meta(x)
    n, c1, h, w, _ = x.shape
    pad = kernel // 2
    return x.new_empty((n, c1, (h + 2 * pad - kernel) // stride + 1, (w + 2 * pad - kernel) // stride + 1, 16))


def _blocked_conv_cuda(x, packed, bias, co, kernel, stride, fp32_output=False, fused=False):
    _require(not fp32_output, "blocked C2f requires FP16 output and fused FP32 SiLU")
    return ops.conv2d(x, packed, bias, co, kernel, stride, silu=fused)


def _blocked_conv_meta(x, packed, bias, co, kernel, stride, fp32_output=False, fused=False):
    _require(not fp32_output, "blocked C2f requires FP16 output and fused FP32 SiLU")
    return _conv_meta(x, packed, bias, co, kernel, stride)


# --------------------------------------------------------------- thin_blocked

def _pack_cuda(x):
    _require(x.dim() == 4 and x.dtype == torch.float16 and x.numel() > 0,
             "expected FP16 NCHW with positive sizes")
    return ops.pack(x)


def _pack_meta(x):
    n, c, h, w = x.shape
    return x.new_empty((n, (c + 15) // 16, h, w, 16))


def _unpack_cuda(x):
    return ops.unpack(x)


def _unpack_meta(x):
    n, c1, h, w, _ = x.shape
    return x.new_empty((n, c1 * 16, h, w))


def register() -> None:
    if _LIBS:
        return
    tb = _lib("thin_backend")
    _register(tb, "add(Tensor x, Tensor y) -> Tensor", _add_cuda, _add_meta)
    _register(tb, "sigmoid(Tensor x) -> Tensor", lambda x: ops.sigmoid(x), _sigmoid_meta)
    _register(tb, "maxpool2d(Tensor x) -> Tensor", _maxpool2d_cuda, lambda x: torch.empty_like(_nchw_meta(x)))
    _register(tb, "upsample_nearest2d(Tensor x) -> Tensor", lambda x: ops.upsample_nearest2d(x),
              _upsample_meta)
    nf = _lib("thin_native_flow")
    _register(nf, "maxpool(Tensor x, int kernel) -> Tensor", lambda x, k: ops.maxpool_blocked(x, k),
              _maxpool_meta)
    _register(nf, "upsample(Tensor x) -> Tensor", lambda x: ops.upsample_blocked(x), _upsample_blocked_meta)
    _register(nf, "detection_select(Tensor decoded, int max_det, bool agnostic=False) -> Tensor",
              _select_cuda, _select_meta)
    _register(nf, "detection_select_trace(Tensor decoded, int max_det, bool agnostic=False) -> Tensor[]",
              _select_trace_cuda, _select_trace_meta)
    _register(nf, "silu_(Tensor(a!) x) -> Tensor(a!)", _silu__cuda, _silu__meta)
    _register(nf, "sppf(Tensor x, int kernel=5) -> Tensor", lambda x, k=5: ops.sppf(x, k), _sppf_meta)
    _register(nf, "softmax(Tensor x, int dim, float scale=1.0, bool half_to_float=False) -> Tensor",
              _softmax_cuda, _softmax_meta)
    _register(nf, "dfl_decode(Tensor box, Tensor cls, int[] heights, int[] widths, float[] strides, "
                  "bool xywh=True) -> Tensor", _decode_cuda, _decode_meta)
    _register(nf, "bias_silu_residual(Tensor x, Tensor bias, Tensor residual) -> Tensor", _bsr_cuda,
              _bsr_meta)
    _register(nf, "conv(Tensor x, Tensor packed, Tensor? bias, int co, int kernel, int stride, bool fused=True, "
                  "bool nchw_output=False) -> Tensor", _conv_cuda, _conv_meta)
    _register(nf, "depthwise(Tensor x, Tensor packed, Tensor? bias, int kernel, int stride, bool fused=True) -> Tensor",
              _depthwise_cuda, _depthwise_meta)
    _register(nf, "pack_input(Tensor x) -> Tensor", _pack_cuda, _pack_meta)
    bl = _lib("thin_blocked")
    _register(bl, "pack(Tensor x) -> Tensor", _pack_cuda, _pack_meta)
    _register(bl, "unpack(Tensor x) -> Tensor", _unpack_cuda, _unpack_meta)
    _register(bl, "conv(Tensor x, Tensor packed, Tensor? bias, int co, int kernel, int stride, "
                  "bool fp32_output=False, bool fused=False) -> Tensor", _blocked_conv_cuda, _blocked_conv_meta)


register()
