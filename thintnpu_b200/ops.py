"""Tensor-level entry points over libttn (PyTorch is only the memory/stream plumbing).

Every function takes CUDA tensors, launches on ``torch.cuda.current_stream()``
and returns new caller-owned tensors (or writes ``out``).  Checks and messages
mirror the reference host code (maxesisnclaw/ThinTNPU backend.cpp, ops.cpp,
flow_ops.cpp, softmax_host.cpp, selection_flow.cpp): failures raise
RuntimeError, never fall back to another implementation.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import TtnTensor, call

_DTYPES = {torch.float16: _lib.F16, torch.float32: _lib.F32}


def _fail(message: str):
    raise RuntimeError(message)


def _require(cond: bool, message: str) -> None:
    if not cond:
        _fail(message)


def _cuda(x: torch.Tensor, what: str) -> None:
    _require(isinstance(x, torch.Tensor) and x.is_cuda, f"{what} requires a CUDA tensor")
    _require(not (x.requires_grad and torch.is_grad_enabled()),
             f"{what} is inference-only; use no_grad/inference_mode")


def desc(x: torch.Tensor) -> TtnTensor:
    """Descriptor of a strided view (data points at element [0,...,0])."""
    dtype = _DTYPES.get(x.dtype)
    _require(dtype is not None, f"unsupported dtype {x.dtype}: float16/float32 only")
    _require(x.dim() <= _lib.MAX_DIMS, f"at most {_lib.MAX_DIMS} dims are supported")
    d = TtnTensor()
    d.data = x.data_ptr() if x.numel() else None
    d.ndim = x.dim()
    d.dtype = dtype
    for i, (s, t) in enumerate(zip(x.shape, x.stride())):
        d.sizes[i] = s
        d.strides[i] = t
    return d


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ref(d: TtnTensor):
    return ctypes.byref(d)


# ------------------------------------------------------------------ elementwise

def silu_(x: torch.Tensor) -> torch.Tensor:
    """In-place SiLU (reference thin_ops::silu_, ops.cpp:498-512)."""
    _cuda(x, "silu_")
    if x.numel():
        d = desc(x)
        call("ttn_silu", _ref(d), _ref(d), stream())
    return x


def silu(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """SiLU into a new tensor (reference aten::silu, aten_adapter.cpp:98-105)."""
    _cuda(x, "silu")
    y = torch.empty_like(x) if out is None else out
    if x.numel():
        call("ttn_silu", _ref(desc(x)), _ref(desc(y)), stream())
    return y


def sigmoid(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sigmoid, bit-equal to CPU eager for fp16 (reference thin::sigmoid, backend.cpp:226-244)."""
    _cuda(x, "sigmoid")
    _require(x.dtype in _DTYPES, "sigmoid supports float32 and float16")
    y = torch.empty_like(x) if out is None else out
    if x.numel():
        call("ttn_sigmoid", _ref(desc(x)), _ref(desc(y)), stream())
    return y


_BINARY = {"sub": _lib.SUB, "mul": _lib.MUL, "div": _lib.DIV, "add": _lib.ADD}


def binary(op: str, x, y, alpha: float = 1.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x (op) alpha*y with broadcasting (reference binary(), ops.cpp:464-497)."""
    code = _BINARY[op]
    if not isinstance(y, torch.Tensor) or (y.dim() == 0 and not y.is_cuda):
        scalar = float(y)
        _cuda(x, op)
        _require(x.dtype in _DTYPES, "binary supports float32/float16")
        if op in ("add", "sub"):
            scalar *= float(alpha)
        z = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
        if x.numel():
            call("ttn_binary_scalar", code, scalar, _ref(desc(x)), _ref(desc(z)), stream())
        return z
    if not isinstance(x, torch.Tensor) or (x.dim() == 0 and not x.is_cuda):
        x = torch.full((), float(x), dtype=y.dtype, device=y.device)
    _cuda(x, op)
    _cuda(y, op)
    _require(x.device == y.device and x.dtype == y.dtype,
             "binary requires matching device, shape and dtype")
    _require(x.dtype in _DTYPES, "binary supports float32/float16")
    shape = torch.broadcast_shapes(x.shape, y.shape)
    xe, ye = x.expand(shape), y.expand(shape)
    z = torch.empty(shape, dtype=x.dtype, device=x.device) if out is None else out
    if z.numel():
        call("ttn_binary", code, float(alpha), _ref(desc(xe)), _ref(desc(ye)), _ref(desc(z)), stream())
    return z


def add_silu(a: torch.Tensor, raw: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """a + SiLU(raw) in one pass (fp16, equal shapes): the C2f bottleneck's activation and
    residual add (ops.cpp:498-512, blocked_c2f.py:20-24), bit-identical to ``silu`` then
    ``add``.  Views that are not rows of aligned contiguous vectors take those two kernels."""
    _cuda(a, "add_silu")
    _cuda(raw, "add_silu")
    _require(a.dtype == raw.dtype == torch.float16 and a.shape == raw.shape and a.device == raw.device,
             "add_silu requires fp16 operands of one shape on one device")
    z = torch.empty_like(a, memory_format=torch.contiguous_format) if out is None else out
    _require(z.shape == a.shape and z.dtype == torch.float16, "add_silu: out must match a")
    if not z.numel():
        return z
    status = _lib.lib().ttn_add_silu_f16(_ref(desc(a)), _ref(desc(raw)), _ref(desc(z)), stream())
    if status == _lib.UNSUPPORTED:
        return binary("add", a, silu(raw), out=z)
    _lib.check("ttn_add_silu_f16", status)
    return z


def add(x, y, alpha: float = 1.0) -> torch.Tensor:
    return binary("add", x, y, alpha)


def sub(x, y, alpha: float = 1.0) -> torch.Tensor:
    return binary("sub", x, y, alpha)


def mul(x, y) -> torch.Tensor:
    return binary("mul", x, y)


def div(x, y) -> torch.Tensor:
    return binary("div", x, y)


def bias_silu_residual(x: torch.Tensor, bias: torch.Tensor, residual: torch.Tensor,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = SiLU(x + bias[c]) + residual over NC1HWC0 fp16 [n, c1, h, w, 16] (one rounding)."""
    for t, name in ((x, "x"), (bias, "bias"), (residual, "residual")):
        _cuda(t, "bias_silu_residual")
        _require(t.dtype == torch.float16 and t.is_contiguous(),
                 f"bias_silu_residual: {name} must be contiguous float16")
    _require(x.dim() == 5 and x.size(-1) == 16, "bias_silu_residual expects NC1HWC0 [n,c1,h,w,16]")
    _require(residual.shape == x.shape, "bias_silu_residual: residual shape differs")
    _require(bias.numel() == x.size(1) * 16, "bias_silu_residual: bias must have c1*16 values")
    y = torch.empty_like(x) if out is None else out
    n, c1, h, w, _ = x.shape
    call("ttn_bias_silu_residual_nc1hwc0_f16", x.data_ptr(), bias.data_ptr(), residual.data_ptr(),
         y.data_ptr(), n, c1, h * w, stream())
    return y


# ------------------------------------------------------------------ data movement

def copy_(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """Device-to-device strided copy (reference thin_ops::copy_strided, ops.cpp:31-84)."""
    _cuda(dst, "copy")
    _cuda(src, "copy")
    _require(dst.shape == src.shape and dst.dtype == src.dtype,
             "copy requires matching sizes and dtype")
    if dst.numel():
        call("ttn_copy", _ref(desc(src)), _ref(desc(dst)), stream())
    return dst


def contiguous(x: torch.Tensor) -> torch.Tensor:
    if x.is_contiguous():
        return x
    return copy_(torch.empty(x.shape, dtype=x.dtype, device=x.device), x)


def cat(tensors: Sequence[torch.Tensor], dim: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """torch.cat semantics, bitwise (reference cat(), ops.cpp:419-462)."""
    tensors = list(tensors)
    _require(len(tensors) > 0, "cat expects a nonempty tensor list")
    reference = tensors[0]
    for t in tensors:
        _cuda(t, "cat")
        _require(t.dim() > 0, "cat cannot concatenate scalar tensors")
        if not (t.dim() == 1 and t.numel() == 0):
            reference = t
    dim = dim % reference.dim()
    sizes = list(reference.shape)
    sizes[dim] = 0
    live = []
    for t in tensors:
        _require(t.device == reference.device and t.dtype == reference.dtype,
                 "cat requires matching device and dtype")
        if t.dim() == 1 and t.numel() == 0:
            continue
        _require(t.dim() == reference.dim(), "cat rank mismatch")
        for d in range(t.dim()):
            _require(d == dim or t.size(d) == reference.size(d),
                     "cat shape mismatch outside concatenation dimension")
        sizes[dim] += t.size(dim)
        if t.numel():
            live.append(t)
    if out is None:
        out = torch.empty(sizes, dtype=reference.dtype, device=reference.device)
    _require(list(out.shape) == sizes, "cat: out has the wrong shape")
    if out.numel() and live:
        descs = (TtnTensor * len(live))(*[desc(t) for t in live])
        call("ttn_cat", len(live), descs, dim, _ref(desc(out)), stream())
    return out


def unpack(x: torch.Tensor, channels: Optional[int] = None, out: Optional[torch.Tensor] = None,
           out_offset: int = 0) -> torch.Tensor:
    """NC1HWC0 [n,c1,h,w,16] -> NCHW [n, channels, h, w] (reference unpack, layout_blocked.h:60-69).

    With ``out`` of shape [n, C, A] the pixels land at columns
    [out_offset, out_offset + h*w) -- the Detect restore writing straight
    into the concatenated [n, no, anchors] head (conv_flow.cpp:87-121)."""
    _cuda(x, "unpack")
    _require(x.dim() == 5 and x.size(4) == 16 and x.dtype == torch.float16 and x.is_contiguous(),
             "expected contiguous FP16 NC1HWC0 with C0=16")
    n, c1, h, w, _ = x.shape
    channels = c1 * 16 if channels is None else channels
    _require(0 < channels <= c1 * 16, "unpack: channels must be in (0, c1*16]")
    if out is None:
        out = torch.empty((n, channels, h, w), dtype=x.dtype, device=x.device)
        bs, cs, base = out.stride(0), out.stride(1), out.data_ptr()
    else:
        _require(out.dim() == 3 and out.size(0) == n and out.size(1) >= channels and out.stride(2) == 1,
                 "unpack: out must be [n, >=channels, anchors] with a unit last stride")
        _require(out_offset + h * w <= out.size(2), "unpack: out_offset + h*w exceeds out")
        bs, cs = out.stride(0), out.stride(1)
        base = out.data_ptr() + out_offset * out.element_size()
    if x.numel():
        call("ttn_nc1hwc0_to_nchw_f16", x.data_ptr(), n, c1, h * w, channels, base, bs, cs, stream())
    return out


def pack(x: torch.Tensor) -> torch.Tensor:
    """NCHW [n,c,h,w] -> NC1HWC0 [n, ceil(c/16), h, w, 16], zero-padded (layout_blocked.h:43-58)."""
    _cuda(x, "pack")
    _require(x.dim() == 4 and x.dtype == torch.float16, "pack expects FP16 NCHW")
    x = contiguous(x)
    n, c, h, w = x.shape
    y = torch.empty((n, (c + 15) // 16, h, w, 16), dtype=x.dtype, device=x.device)
    if y.numel():
        call("ttn_nchw_to_nc1hwc0_f16", x.data_ptr(), n, c, h * w, y.data_ptr(), stream())
    return y


# ------------------------------------------------------------------ spatial

def _blocked(x: torch.Tensor, what: str) -> None:
    _cuda(x, what)
    _require(x.dim() == 5 and x.size(4) == 16 and x.dtype == torch.float16 and x.is_contiguous()
             and (x.data_ptr() % 16 == 0),
             "expected aligned contiguous FP16 NC1HWC0 input, C0=16")
    _require(x.size(1) > 0 and x.size(2) > 0 and x.size(3) > 0,
             "blocked spatial operators require positive C1/H/W")


def upsample_blocked(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Nearest 2x on NC1HWC0 (reference blocked_flow::upsample, flow_ops.cpp:233-252).

    ``x`` and ``out`` may be batch-strided views (each image dense), e.g. a slice
    of a concat buffer along C1."""
    _cuda(x, "upsample")
    _require(x.dim() == 5 and x.size(4) == 16 and x.dtype == torch.float16,
             "expected aligned contiguous FP16 NC1HWC0 input, C0=16")
    _require(x.size(1) > 0 and x.size(2) > 0 and x.size(3) > 0,
             "blocked spatial operators require positive C1/H/W")
    n, c1, h, w, _ = x.shape
    y = torch.empty((n, c1, 2 * h, 2 * w, 16), dtype=x.dtype, device=x.device) if out is None else out
    _require(tuple(y.shape) == (n, c1, 2 * h, 2 * w, 16), "upsample: bad out shape")
    _require(_image_dense(x) and _image_dense(y), "upsample: each image must be dense")
    call("ttn_upsample2x_nc1hwc0_f16", x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), n, c1, h, w,
         stream())
    return y


def _image_dense(t: torch.Tensor) -> bool:
    """True when every image (dims 1..) of t is a dense row-major block."""
    expect = 1
    for d in range(t.dim() - 1, 0, -1):
        if t.size(d) != 1 and t.stride(d) != expect:
            return False
        expect *= t.size(d)
    return True


def maxpool_blocked(x: torch.Tensor, kernel: int) -> torch.Tensor:
    """k x k / s1 / p k//2 max-pool on NC1HWC0 (reference blocked_flow::maxpool, flow_ops.cpp:208-231)."""
    _blocked(x, "maxpool")
    _require(kernel >= 1 and kernel % 2 == 1, "maxpool kernel must be a positive odd integer")
    n, c1, h, w, _ = x.shape
    y = torch.empty_like(x)
    call("ttn_maxpool", _lib.NC1HWC0, _lib.F16, int(kernel), x.data_ptr(), y.data_ptr(), n, c1, h, w,
         stream())
    return y


def sppf(x: torch.Tensor, kernel: int = 5, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """cat(x, p1, p2, p3) along C1 with three chained max-pools, one kernel (SPPF tail)."""
    _blocked(x, "sppf")
    _require(kernel >= 1 and kernel % 2 == 1, "maxpool kernel must be a positive odd integer")
    n, c1, h, w, _ = x.shape
    y = torch.empty((n, 4 * c1, h, w, 16), dtype=x.dtype, device=x.device) if out is None else out
    call("ttn_sppf_f16", x.data_ptr(), y.data_ptr(), n, c1, h, w, int(kernel), stream())
    return y


def _nchw(x: torch.Tensor, what: str) -> None:
    _cuda(x, what)
    _require(x.dim() == 4 and x.is_contiguous(), f"{what} requires contiguous NCHW")
    _require(x.dtype in _DTYPES, f"{what} supports float32/float16")
    _require(x.size(1) > 0 and x.size(2) > 0 and x.size(3) > 0, "C, H, W must be positive")


def upsample_nearest2d(x: torch.Tensor) -> torch.Tensor:
    """Nearest 2x on NCHW (reference thin::upsample_nearest2d, backend.cpp:266-286)."""
    _nchw(x, "upsample_nearest2d")
    n, c, h, w = x.shape
    y = torch.empty((n, c, 2 * h, 2 * w), dtype=x.dtype, device=x.device)
    if y.numel():
        call("ttn_upsample2x", _lib.NCHW, _DTYPES[x.dtype], x.data_ptr(), y.data_ptr(), n, c, h, w,
             stream())
    return y


def maxpool2d(x: torch.Tensor, kernel: int = 5) -> torch.Tensor:
    """k x k / s1 / p k//2 max-pool on NCHW (reference thin::maxpool2d, backend.cpp:245-265)."""
    _nchw(x, "maxpool2d")
    n, c, h, w = x.shape
    y = torch.empty_like(x)
    if y.numel():
        call("ttn_maxpool", _lib.NCHW, _DTYPES[x.dtype], int(kernel), x.data_ptr(), y.data_ptr(), n, c,
             h, w, stream())
    return y


# ------------------------------------------------------------------ softmax / decode

def softmax(x: torch.Tensor, dim: int = -1, half_to_float: bool = False, scale: float = 1.0,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(x * scale) over ``dim`` (reference thin_softmax::softmax, softmax_host.cpp:51-89).

    scale != 1 rounds x*scale to x's dtype first, like the separate fp16
    multiply before the attention softmax (whole_blocked.py:101-102)."""
    _cuda(x, "softmax")
    _require(x.dtype in _DTYPES, "softmax supports float32/float16")
    _require(not half_to_float or x.dtype == torch.float16, "half_to_float requires float16 input")
    dim = dim % x.dim() if x.dim() else 0
    dtype = torch.float32 if half_to_float else x.dtype
    y = torch.empty(x.shape, dtype=dtype, device=x.device) if out is None else out
    if x.numel():
        call("ttn_softmax", _ref(desc(x)), dim, float(scale), _ref(desc(y)), stream())
    return y


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
              out: Optional[torch.Tensor] = None, prescale: bool = False) -> torch.Tensor:
    """Fused C2PSA attention: v @ softmax((q^T @ k) * scale)^T per (image, head),
    rounding as the reference's separate fp16 ops do (whole_blocked.py:91-103);
    ``prescale`` is the reference's ``attention_scale_before_matmul`` order
    (YOLO26): ``(q * scale)^T @ k`` with the scaled query rounded to fp16.

    q, k: fp16 [B, heads, key_dim, N] and v: [B, heads, head_dim, N] views with
    the token dim contiguous -- e.g. the split of the qkv conv output
    ``qkv.view(B, heads, 2*key_dim + head_dim, N).split(...)``.  Returns (or
    fills) out [B, heads, head_dim, N]."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _cuda(t, "attention")
        _require(t.dtype == torch.float16 and t.dim() == 4 and t.stride(3) == 1,
                 f"attention: {name} must be fp16 [B, heads, C, N] with the token dim contiguous")
    b, h, kd, n = q.shape
    hd = v.size(2)
    _require(tuple(k.shape) == (b, h, kd, n) and tuple(v.shape[:2]) == (b, h) and v.size(3) == n,
             "attention: q, k, v shapes disagree")
    if out is None:
        out = torch.empty((b, h, hd, n), dtype=torch.float16, device=q.device)
    _require(tuple(out.shape) == (b, h, hd, n) and out.dtype == torch.float16 and out.stride(3) == 1,
             "attention: out must be fp16 [B, heads, head_dim, N] with the token dim contiguous")

    def strides(t):
        return (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))

    if q.numel() and v.numel():
        call("ttn_attention_f16", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, h, n, kd, hd,
             strides(q), strides(k), strides(v), strides(out), float(scale),
             _lib.ATTENTION_PRESCALE if prescale else 0, stream())
    return out


def attention_fault() -> int:
    """Reads and clears the attention kernel's fault word (0 = no launch gave up)."""
    word = ctypes.c_uint32(0)
    call("ttn_attention_fault_f16", ctypes.byref(word))
    return int(word.value)


def conv2d_pack_weights(w: torch.Tensor) -> torch.Tensor:
    """OIHW fp16 weights [co, ci, k, k] (k = 1, 3 or 6) on the GPU -> the reference's
    prepared layout [ceil(ci/16), k*k, co64, 16] (conv_img.cpp:321-383)."""
    _cuda(w, "conv2d_pack_weights")
    _require(w.dtype == torch.float16 and w.dim() == 4 and w.size(2) == w.size(3) and w.is_contiguous(),
             "conv2d_pack_weights: expected contiguous fp16 OIHW weights")
    co, ci, k, _ = w.shape
    packed = torch.empty(((ci + 15) // 16, k * k, (co + 63) // 64 * 64, 16), dtype=torch.float16, device=w.device)
    call("ttn_conv2d_pack_weights_f16", w.data_ptr(), co, ci, k, packed.data_ptr(), stream())
    return packed


def conv2d(x: torch.Tensor, packed: torch.Tensor, bias: Optional[torch.Tensor], co: int, kernel: int,
           stride: int = 1, silu: bool = True, nchw: bool = False,
           out: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The reference's fused convolution (thin_native_flow::conv, conv_flow.cpp:594-646) on
    the tensor cores: x NC1HWC0 fp16 [B, C1, H, W, 16] (images may be strided), packed
    weights from ``conv2d_pack_weights``, bias fp16 [co] or None; returns (or fills)
    NC1HWC0 [B, co/16, OH, OW, 16], or NCHW [B, co, OH, OW] with ``nchw``.  ``out`` may
    be a batch-strided view, e.g. a channel slice of a concat buffer.  ``residual``
    (NC1HWC0, the output's shape, dense images; may be ``out`` itself) is added after
    the epilogue as the reference's residual bottleneck does (blocked_c2f.py:20-24):
    fp16(residual + y), bit-identical to the conv followed by the fp16 add."""
    _cuda(x, "conv2d")
    _require(x.dtype == torch.float16 and x.dim() == 5 and x.size(4) == 16 and x[0].is_contiguous(),
             "conv2d: x must be fp16 NC1HWC0 [B, C1, H, W, 16] with dense images")
    b, c1, h, w, _ = x.shape
    _require(packed.dtype == torch.float16 and packed.is_contiguous() and packed.dim() == 4 and
             tuple(packed.shape) == (c1, kernel * kernel, (co + 63) // 64 * 64, 16),
             "conv2d: packed weights must be [C1, k*k, co64, 16] (conv2d_pack_weights)")
    if bias is not None:
        _require(bias.dtype == torch.float16 and bias.is_contiguous() and bias.numel() >= co,
                 "conv2d: bias must be contiguous fp16 with at least co elements")
    pad = (kernel - 1) // 2
    oh, ow = (h + 2 * pad - kernel) // stride + 1, (w + 2 * pad - kernel) // stride + 1
    shape = (b, co, oh, ow) if nchw else (b, co // 16, oh, ow, 16)
    if out is None:
        out = torch.empty(shape, dtype=torch.float16, device=x.device)
    _require(tuple(out.shape) == shape and out.dtype == torch.float16 and out[0].is_contiguous(),
             f"conv2d: out must be fp16 {shape} with dense images")
    flags = (_lib.CONV_SILU if silu else 0) | (_lib.CONV_NCHW if nchw else 0)
    x_bs, out_bs = x.stride(0) if b > 1 else c1 * h * w * 16, out.stride(0) if b > 1 else out[0].numel()
    bias_ptr = None if bias is None else bias.data_ptr()
    if residual is None:
        call("ttn_conv2d_nc1hwc0_f16", x.data_ptr(), b, c1, h, w, x_bs, packed.data_ptr(), bias_ptr, co, kernel,
             stride, flags, out.data_ptr(), out_bs, stream())
        return out
    _cuda(residual, "conv2d")
    _require(not nchw, "conv2d: the residual needs NC1HWC0 output")
    _require(tuple(residual.shape) == shape and residual.dtype == torch.float16 and residual[0].is_contiguous(),
             f"conv2d: residual must be fp16 {shape} with dense images")
    call("ttn_conv2d_residual_nc1hwc0_f16", x.data_ptr(), b, c1, h, w, x_bs, packed.data_ptr(), bias_ptr, co,
         kernel, stride, flags, residual.data_ptr(), residual.stride(0) if b > 1 else residual[0].numel(),
         out.data_ptr(), out_bs, stream())
    return out


def depthwise_pack_weights(w: torch.Tensor) -> torch.Tensor:
    """Depthwise weights [C, 1, k, k] fp16 -> [C/16, k, k, 16] (verify_depthwise_flow.py:27-30)."""
    c, one, k, k2 = w.shape
    _require(one == 1 and k == k2 and c % 16 == 0, "depthwise_pack_weights: expected [C, 1, k, k] with C % 16 == 0")
    return w.reshape(c // 16, 16, k, k).permute(0, 2, 3, 1).contiguous()


def depthwise(x: torch.Tensor, packed: torch.Tensor, bias: Optional[torch.Tensor], kernel: int, stride: int = 1,
              silu: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The reference's depthwise conv (thin_native_flow::depthwise, depthwise_flow.cpp:164-226)
    over NC1HWC0 fp16 [B, C1, H, W, 16]; packed weights [C1, k, k, 16]; bias fp16 [16*C1]
    or None; returns (or fills) NC1HWC0 [B, C1, OH, OW, 16]."""
    _cuda(x, "depthwise")
    _require(x.dtype == torch.float16 and x.dim() == 5 and x.size(4) == 16 and x[0].is_contiguous(),
             "depthwise: x must be fp16 NC1HWC0 [B, C1, H, W, 16] with dense images")
    b, c1, h, w, _ = x.shape
    _require(packed.dtype == torch.float16 and packed.is_contiguous() and
             tuple(packed.shape) == (c1, kernel, kernel, 16), "depthwise: packed weights must be [C1, k, k, 16]")
    if bias is not None:
        _require(bias.dtype == torch.float16 and bias.is_contiguous() and bias.numel() == 16 * c1,
                 "depthwise: bias must be contiguous fp16 [16*C1]")
    pad = kernel // 2
    oh, ow = (h + 2 * pad - kernel) // stride + 1, (w + 2 * pad - kernel) // stride + 1
    shape = (b, c1, oh, ow, 16)
    if out is None:
        out = torch.empty(shape, dtype=torch.float16, device=x.device)
    _require(tuple(out.shape) == shape and out.dtype == torch.float16 and out[0].is_contiguous(),
             f"depthwise: out must be fp16 {shape} with dense images")
    call("ttn_depthwise_nc1hwc0_f16", x.data_ptr(), b, c1, h, w, x.stride(0) if b > 1 else x[0].numel(),
         packed.data_ptr(), None if bias is None else bias.data_ptr(), kernel, stride,
         _lib.CONV_SILU if silu else 0, out.data_ptr(), out.stride(0) if b > 1 else out[0].numel(), stream())
    return out


def conv2d_fault() -> int:
    """Reads and clears the convolution kernel's fault word (0 = no launch gave up)."""
    word = ctypes.c_uint32(0)
    call("ttn_conv2d_fault_f16", ctypes.byref(word))
    return int(word.value)


def dfl_decode(box: torch.Tensor, cls: torch.Tensor, shapes: Sequence[tuple],
               strides: Sequence[float], xywh: bool = True,
               out: Optional[torch.Tensor] = None, distances: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Detect decode: DFL(16) softmax + expectation, anchor decode, sigmoid(cls).

    box [n, 64, a] and cls [n, nc, a] fp16 logits (any batch/channel strides,
    unit anchor stride); shapes = [(h, w)] per level; strides per level.
    Returns [n, 4+nc, a] = cat(boxes*stride, sigmoid(cls)) (whole_blocked.py:118-146).
    ``distances`` (fp16 [n, 4, a], contiguous) also receives the DFL expectations
    the boxes were decoded from (the trace entry point)."""
    for t, name in ((box, "box"), (cls, "cls")):
        _cuda(t, "dfl_decode")
        _require(t.dtype == torch.float16 and t.dim() == 3 and t.stride(2) == 1,
                 f"dfl_decode: {name} must be fp16 [n, c, anchors] with unit anchor stride")
    n, c, a = box.shape
    _require(c == 64, "dfl_decode: box must have 4*16 channels")
    _require(cls.size(0) == n and cls.size(2) == a, "dfl_decode: box/cls shapes differ")
    levels = len(shapes)
    _require(levels == len(strides) and levels > 0, "dfl_decode: one stride per level")
    _require(sum(h * w for h, w in shapes) == a, "dfl_decode: level sizes do not sum to anchors")
    nc = cls.size(1)
    heights = (ctypes.c_int64 * levels)(*[int(h) for h, _ in shapes])
    widths = (ctypes.c_int64 * levels)(*[int(w) for _, w in shapes])
    strides_c = (ctypes.c_float * levels)(*[float(s) for s in strides])
    y = torch.empty((n, 4 + nc, a), dtype=torch.float16, device=box.device) if out is None else out
    _require(y.is_contiguous() and tuple(y.shape) == (n, 4 + nc, a), "dfl_decode: bad out")
    if distances is None:
        call("ttn_dfl_decode_f16", box.data_ptr(), box.stride(0), box.stride(1), cls.data_ptr(),
             cls.stride(0), cls.stride(1), n, nc, levels, heights, widths, strides_c, int(bool(xywh)),
             y.data_ptr(), stream())
        return y
    _cuda(distances, "dfl_decode")
    _require(distances.dtype == torch.float16 and distances.is_contiguous() and tuple(distances.shape) == (n, 4, a),
             "dfl_decode: distances must be contiguous fp16 [n, 4, anchors]")
    call("ttn_dfl_decode_trace_f16", box.data_ptr(), box.stride(0), box.stride(1), cls.data_ptr(),
         cls.stride(0), cls.stride(1), n, nc, levels, heights, widths, strides_c, int(bool(xywh)),
         y.data_ptr(), distances.data_ptr(), stream())
    return y


# ------------------------------------------------------------------ selection

TRACE_NAMES = ("output", "class_max", "stage1_indices", "gathered_scores", "top_values",
               "stage2_indices", "anchor_indices", "labels")


def workspace_size(batch: int, anchors: int, classes: int, max_det: int, flags: int) -> int:
    return int(_lib.lib().ttn_select_workspace_size(batch, anchors, classes, max_det, flags))


def detection_select(decoded: torch.Tensor, max_det: int, agnostic: bool = False, *,
                     nan_last: bool = False, apply_sigmoid: bool = False, trace: bool = False,
                     workspace: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
    """YOLO26 stable top-k selection (reference detection_selection::run, selection_flow.cpp:429-491).

    decoded: fp16 [B, A, 4+nc] view (boxes then scores).  Returns FP32
    [B, k, 6] rows, or with ``trace`` the 8 stage tensors of
    detection_select_trace in TRACE_NAMES order."""
    _cuda(decoded, "detection_select")
    _require(decoded.dtype == torch.float16 and decoded.dim() == 3,
             "detection_select expects inference-only device FP16 [B,A,4+nc]")
    _require(decoded.size(2) > 4 and max_det >= 0, "detection_select requires nc > 0 and max_det >= 0")
    b, a, channels = decoded.shape
    nc, k = channels - 4, min(int(max_det), a)
    flags = ((_lib.SELECT_AGNOSTIC if agnostic else 0) | (_lib.SELECT_NAN_LAST if nan_last else 0)
             | (_lib.SELECT_SIGMOID if apply_sigmoid else 0))
    dev = decoded.device
    output = torch.empty((b, k, 6), dtype=torch.float32, device=dev) if out is None else out
    _require(tuple(output.shape) == (b, k, 6) and output.dtype == torch.float32 and output.is_contiguous(),
             "detection_select: out must be contiguous float32 [B, k, 6]")
    tr = _lib.SelectTrace()
    tensors = None
    if trace:
        tensors = dict(
            class_max=torch.empty((b, a), dtype=torch.float16, device=dev),
            stage1_indices=torch.empty((b, k), dtype=torch.int64, device=dev),
            gathered_scores=torch.empty((b, 0 if agnostic else k, nc), dtype=torch.float16, device=dev),
            top_values=torch.empty((b, k), dtype=torch.float16, device=dev),
            stage2_indices=torch.empty((b, 0 if agnostic else k), dtype=torch.int64, device=dev),
            anchor_indices=torch.empty((b, k), dtype=torch.int64, device=dev),
            labels=torch.empty((b, k), dtype=torch.int64, device=dev))
        for name, t in tensors.items():
            setattr(tr, name, t.data_ptr() if t.numel() else None)
    if b and a and (k or trace):
        need = workspace_size(b, a, nc, k, flags)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        call("ttn_select_f16", _ref(desc(decoded)), k, flags, workspace.data_ptr(), workspace.numel(),
             output.data_ptr() if output.numel() else None, ctypes.byref(tr), stream())
    if not trace:
        return output
    return [output] + [tensors[name] for name in TRACE_NAMES[1:]]
