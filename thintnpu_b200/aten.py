"""ATen routing: send the op pass's ATen calls on CUDA tensors to libttn.

The reference overrides these ATen ops for its PrivateUse1 device
(aten_adapter.cpp:106-112, ops.cpp:513-524, softmax_host.cpp:90-92,
backend.cpp:357-361).  On CUDA tensors, which PyTorch's own kernels also serve,
the routing is opt-in: a dispatch mode, active inside ``with aten_routing():``
or after ``enable_aten_routing()`` (``import thin_backend`` turns it on only
when ``THIN_BACKEND_ATEN=1``), so code that does not ask for it pays nothing:

    silu, silu_, sigmoid, add/sub/mul/div.Tensor (and .Scalar), cat, _softmax,
    max_pool2d and max_pool2d_with_indices (k5/s1/p2 only; indices are a zero
    placeholder), upsample_nearest2d (2x only), copy_ (device to device, same
    dtype), convolution (fp16, k1/p0 stride 1 or k3/p1 stride 1/2, groups 1: the
    tensor-core conv of ttn_conv2d_nc1hwc0_f16 with NCHW output)

for float16/float32 CUDA tensors.  Calls with unsupported arguments raise, as
the reference's TORCH_CHECKs do; other dtypes, devices and ops are left to
PyTorch.  ``THIN_ATEN_TRACE=1`` logs each routed call (aten_adapter.cpp:25-29).
"""
from __future__ import annotations

import os
import sys
from contextlib import contextmanager
from typing import Dict

import torch
from torch.utils._python_dispatch import TorchDispatchMode

from . import ops

aten = torch.ops.aten
_FLOATS = (torch.float16, torch.float32)
ROUTED: Dict[str, int] = {}


def _trace(name: str, target: str) -> None:
    ROUTED[name] = ROUTED.get(name, 0) + 1
    if os.environ.get("THIN_ATEN_TRACE") == "1":
        sys.stderr.write(f"THIN_ATEN {name} -> {target} device=cuda\n")


def _ours(*tensors) -> bool:
    seen = False
    for t in tensors:
        if isinstance(t, torch.Tensor):
            if t.dim() == 0 and not t.is_cuda:
                continue  # CPU scalar operand
            if not t.is_cuda or t.dtype not in _FLOATS:
                return False
            seen = True
    return seen


def _square(values, name):
    values = list(values)
    if len(values) not in (1, 2) or (len(values) == 2 and values[0] != values[1]):
        raise RuntimeError(f"thin aten: asymmetric or malformed {name} is unsupported")
    return values[0]


def _binary(op):
    def run(x, y, alpha=1):
        _trace(f"aten::{op}", f"ttn_binary({op})")
        return ops.binary(op, x, y, alpha)
    return run


def _maxpool(x, kernel_size, stride=(), padding=0, dilation=1, ceil_mode=False):
    k = _square(kernel_size, "kernel_size")
    s = _square(stride, "stride") if len(list(stride)) else k
    p = _square(padding if isinstance(padding, (list, tuple)) else [padding], "padding")
    d = _square(dilation if isinstance(dilation, (list, tuple)) else [dilation], "dilation")
    if not (k == 5 and s == 1 and p == 2 and d == 1 and not ceil_mode):
        raise RuntimeError("thin aten maxpool supports only k5/s1/p2/d1, ceil_mode=False")
    _trace("aten::max_pool2d_with_indices", "ttn_maxpool (indices=zeros placeholder)")
    values = ops.maxpool2d(ops.contiguous(x), 5)
    return values, torch.zeros(values.shape, dtype=torch.int64, device=values.device)


def _upsample(x, output_size, scales_h=None, scales_w=None):
    if not (x.dim() == 4 and len(output_size) == 2 and output_size[0] == 2 * x.size(2)
            and output_size[1] == 2 * x.size(3)):
        raise RuntimeError("thin aten nearest2d requires a 2x output size")
    for s in (scales_h, scales_w):
        if s is not None and s != 2.0:
            raise RuntimeError("thin aten nearest2d supports scale=2 only")
    _trace("aten::upsample_nearest2d", "ttn_upsample2x")
    return ops.upsample_nearest2d(ops.contiguous(x))


class AtenRouting(TorchDispatchMode):
    """Dispatch mode routing the op pass's ATen calls on CUDA float tensors to libttn."""

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        handler = _HANDLERS.get(func)
        if handler is not None:
            routed = handler(args, kwargs)
            if routed is not NotImplemented:
                return routed
        return func(*args, **kwargs)


def _h_silu(args, kwargs):
    if not _ours(args[0]):
        return NotImplemented
    _trace("aten::silu", "ttn_silu")
    return ops.silu(args[0])


def _h_silu_(args, kwargs):
    if not _ours(args[0]):
        return NotImplemented
    _trace("aten::silu_", "ttn_silu (in place)")
    return ops.silu_(args[0])


def _h_sigmoid(args, kwargs):
    if not _ours(args[0]):
        return NotImplemented
    _trace("aten::sigmoid", "ttn_sigmoid")
    return ops.sigmoid(args[0])


def _h_binary(op, scalar=False):
    def handler(args, kwargs):
        x, y = args[0], args[1]
        if not _ours(x, y if isinstance(y, torch.Tensor) else None):
            return NotImplemented
        if isinstance(y, torch.Tensor) and y.is_cuda and y.dtype != x.dtype:
            return NotImplemented
        alpha = kwargs.get("alpha", args[2] if len(args) > 2 else 1)
        return _binary(op)(x, y, alpha)
    return handler


def _h_cat(args, kwargs):
    tensors = list(args[0])
    dim = kwargs.get("dim", args[1] if len(args) > 1 else 0)
    live = [t for t in tensors if not (t.dim() == 1 and t.numel() == 0)]
    if not live or not _ours(*live) or len({t.dtype for t in live}) != 1:
        return NotImplemented
    _trace("aten::cat", "ttn_cat")
    return ops.cat(tensors, dim)


def _h_softmax(args, kwargs):
    x, dim, half_to_float = args[0], args[1], args[2]
    if not _ours(x):
        return NotImplemented
    _trace("aten::_softmax", "ttn_softmax")
    return ops.softmax(x, dim, half_to_float=bool(half_to_float))


def _h_softmax_int(args, kwargs):
    x, dim = args[0], args[1]
    dtype = kwargs.get("dtype", args[2] if len(args) > 2 else None)
    if not _ours(x):
        return NotImplemented
    if dtype is not None and dtype != x.dtype and not (dtype == torch.float32 and x.dtype == torch.float16):
        return NotImplemented
    _trace("aten::_softmax", "ttn_softmax")
    return ops.softmax(x, dim, half_to_float=dtype is not None and dtype != x.dtype)


def _h_maxpool(args, kwargs):
    if not _ours(args[0]):
        return NotImplemented
    return _maxpool(*args, **kwargs)


def _h_maxpool_values(args, kwargs):
    if not _ours(args[0]):
        return NotImplemented
    return _maxpool(*args, **kwargs)[0]


def _h_upsample(args, kwargs):
    if not _ours(args[0]):
        return NotImplemented
    return _upsample(*args, **kwargs)


def _h_upsample_vec(args, kwargs):
    x = args[0]
    if not _ours(x):
        return NotImplemented
    output_size = kwargs.get("output_size", args[1] if len(args) > 1 else None)
    scales = kwargs.get("scale_factors", args[2] if len(args) > 2 else None)
    if output_size is None:
        if scales is None or len(scales) != 2 or any(float(s) != 2.0 for s in scales):
            raise RuntimeError("thin aten nearest2d supports scale=2 only")
        output_size = [2 * x.size(2), 2 * x.size(3)]
    return _upsample(x, list(output_size))


_PACKED_WEIGHTS: Dict[tuple, torch.Tensor] = {}


def _packed_weight(w: torch.Tensor) -> torch.Tensor:
    """The prepared conv layout of an OIHW weight, built once per (storage,
    version, shape) and kept while that weight is unchanged."""
    try:
        version = w._version
    except RuntimeError:  # an inference tensor has no version counter: pack every call
        return ops.conv2d_pack_weights(ops.contiguous(w))
    key = (w.data_ptr(), version, tuple(w.shape), tuple(w.stride()))
    packed = _PACKED_WEIGHTS.get(key)
    if packed is None:
        if len(_PACKED_WEIGHTS) > 256:
            _PACKED_WEIGHTS.clear()
        packed = _PACKED_WEIGHTS[key] = ops.conv2d_pack_weights(ops.contiguous(w))
    return packed


def _h_convolution(args, kwargs):
    names = ("input", "weight", "bias", "stride", "padding", "dilation", "transposed", "output_padding", "groups")
    a = dict(zip(names, args), **kwargs)
    x, w, bias = a["input"], a["weight"], a.get("bias")
    if not (_ours(x, w) and x.dtype == torch.float16 and w.dtype == torch.float16):
        return NotImplemented
    if bias is not None and not (_ours(bias) and bias.dtype == torch.float16):
        return NotImplemented
    if a["transposed"] or a["groups"] != 1:
        raise RuntimeError("thin aten convolution: transposed/groups are unsupported")
    if x.dim() != 4 or w.dim() != 4:
        raise RuntimeError("thin aten convolution requires 2D NCHW/OIHW")
    s, p = _square(a["stride"], "stride"), _square(a["padding"], "padding")
    if _square(a["dilation"], "dilation") != 1 or any(v != 0 for v in a["output_padding"]):
        raise RuntimeError("thin aten convolution requires dilation=1 and output_padding=0")
    k = w.size(2)
    if not ((k == 1 and p == 0 and s == 1) or (k == 3 and w.size(3) == 3 and p == 1 and s in (1, 2))):
        raise RuntimeError("thin aten convolution supports only k1/p0 stride 1 or k3/p1 stride 1/2")
    _trace("aten::convolution", "ttn_conv2d_nc1hwc0_f16 (NCHW output)")
    co = w.size(0)
    return ops.conv2d(ops.pack(x), _packed_weight(w), None if bias is None else ops.contiguous(bias), co, k, s,
                      silu=False, nchw=True)


def _h_conv2d(args, kwargs):
    """aten::conv2d (what nn.Conv2d / F.conv2d reach first): the convolution above."""
    names = ("input", "weight", "bias", "stride", "padding", "dilation", "groups")
    a = dict(zip(names, args), **kwargs)
    pair = lambda v, d: list(v) if isinstance(v, (list, tuple)) else [v if v is not None else d]
    return _h_convolution((a["input"], a["weight"], a.get("bias"), pair(a.get("stride", 1), 1),
                           pair(a.get("padding", 0), 0), pair(a.get("dilation", 1), 1), False, [0, 0],
                           a.get("groups", 1)), {})


def _h_copy(args, kwargs):
    dst, src = args[0], args[1]
    if not (_ours(dst, src) and dst.dtype == src.dtype and dst.shape == src.shape and dst.device == src.device):
        return NotImplemented
    _trace("aten::copy_", "ttn_copy")
    return ops.copy_(dst, src)


_HANDLERS = {
    aten.silu.default: _h_silu,
    aten.silu_.default: _h_silu_,
    aten.sigmoid.default: _h_sigmoid,
    aten.add.Tensor: _h_binary("add"),
    aten.sub.Tensor: _h_binary("sub"),
    aten.mul.Tensor: _h_binary("mul"),
    aten.div.Tensor: _h_binary("div"),
    aten.add.Scalar: _h_binary("add"),
    aten.sub.Scalar: _h_binary("sub"),
    aten.mul.Scalar: _h_binary("mul"),
    aten.div.Scalar: _h_binary("div"),
    aten.cat.default: _h_cat,
    aten._softmax.default: _h_softmax,
    aten.softmax.int: _h_softmax_int,
    aten.max_pool2d_with_indices.default: _h_maxpool,
    aten.max_pool2d.default: _h_maxpool_values,
    aten.upsample_nearest2d.default: _h_upsample,
    aten.upsample_nearest2d.vec: _h_upsample_vec,
    aten.copy_.default: _h_copy,
    aten.convolution.default: _h_convolution,
    aten.conv2d.default: _h_conv2d,
}


@contextmanager
def aten_routing():
    """Route the op pass's ATen calls on CUDA float tensors to libttn inside the block."""
    with AtenRouting():
        yield


_GLOBAL = None


def enable_aten_routing() -> None:
    """Route for the rest of the process (the reference's import-time behaviour)."""
    global _GLOBAL
    if _GLOBAL is None:
        _GLOBAL = AtenRouting()
        _GLOBAL.__enter__()


def disable_aten_routing() -> None:
    global _GLOBAL
    if _GLOBAL is not None:
        _GLOBAL.__exit__(None, None, None)
        _GLOBAL = None
