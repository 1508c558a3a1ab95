"""PyTorch CPU eager restatements of the op-pass ops (test infrastructure only).

Each function runs on CPU tensors and returns what the reference's own
verification scripts compare against.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch
import torch.nn.functional as F


def to_blocked(x: torch.Tensor) -> torch.Tensor:
    """NCHW [n, c, h, w] -> NC1HWC0 [n, c/16, h, w, 16] (verify_flow_ops.py:13-16, any n)."""
    n, c, h, w = x.shape
    assert c % 16 == 0
    return x.reshape(n, c // 16, 16, h, w).permute(0, 1, 3, 4, 2).contiguous()


def from_blocked(y: torch.Tensor) -> torch.Tensor:
    """NC1HWC0 -> NCHW (verify_flow_ops.py:19-22, any n)."""
    n, c1, h, w, c0 = y.shape
    assert c0 == 16
    return y.permute(0, 1, 4, 2, 3).reshape(n, c1 * 16, h, w).contiguous()


def pack_padded(x: torch.Tensor) -> torch.Tensor:
    """NCHW -> NC1HWC0 with the channel tail zero-padded to 16 (pack_input_channels,
    conv_flow.cpp:406-458)."""
    n, c, h, w = x.shape
    c1 = (c + 15) // 16
    padded = torch.zeros((n, c1 * 16, h, w), dtype=x.dtype)
    padded[:, :c] = x
    return to_blocked(padded)


def silu(x: torch.Tensor) -> torch.Tensor:
    """CPU eager SiLU (elementwise.cpp:71-86 computes the same x/(1+exp(-x)) in FP32)."""
    return F.silu(x)


def sigmoid(x: torch.Tensor) -> torch.Tensor:
    return torch.sigmoid(x)


def binary(op: str, x: torch.Tensor, y, alpha: float = 1.0) -> torch.Tensor:
    """CPU eager add/sub/mul/div (verify_ops.py:68-80)."""
    if op == "add":
        return torch.add(x, y, alpha=alpha)
    if op == "sub":
        return torch.sub(x, y, alpha=alpha)
    return getattr(torch, op)(x, y)


def bias_silu_residual(x: torch.Tensor, bias: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """y = SiLU(x + b) + r in FP32 eager, one rounding to fp16.

    x, residual: NC1HWC0 [n, c1, h, w, 16]; bias [c1*16] indexed b[c1*16 + c0]."""
    b = bias.float().view(1, x.size(1), 1, 1, 16)
    return (F.silu(x.float() + b) + residual.float()).half()


def upsample_blocked(x: torch.Tensor) -> torch.Tensor:
    """Nearest 2x on NC1HWC0 via F.interpolate (verify_flow_ops.py:38-39)."""
    return to_blocked(F.interpolate(from_blocked(x).float(), scale_factor=2, mode="nearest").to(x.dtype))


def maxpool_blocked(x: torch.Tensor, kernel: int) -> torch.Tensor:
    """k/s1/p k//2 max-pool on NC1HWC0 via F.max_pool2d in FP32 (verify_flow_ops.py:25-27)."""
    pooled = F.max_pool2d(from_blocked(x).float(), kernel, stride=1, padding=kernel // 2)
    return to_blocked(pooled.to(x.dtype))


def maxpool_nchw(x: torch.Tensor, kernel: int = 5) -> torch.Tensor:
    """thin_backend::maxpool2d oracle (verify_all.py:82-87)."""
    return F.max_pool2d(x.float(), kernel, 1, kernel // 2).to(x.dtype)


def upsample_nchw(x: torch.Tensor) -> torch.Tensor:
    """thin_backend::upsample_nearest2d oracle (verify_all.py:88-94)."""
    return F.interpolate(x.float(), scale_factor=2, mode="nearest").to(x.dtype)


def sppf(x: torch.Tensor, kernel: int = 5) -> torch.Tensor:
    """SPPF tail: cat(x, p1, p2, p3) along C1, each p a chained max-pool."""
    parts = [x]
    for _ in range(3):
        parts.append(maxpool_blocked(parts[-1], kernel))
    return torch.cat(parts, 1)


def unpack(x: torch.Tensor, channels: int) -> torch.Tensor:
    """NC1HWC0 -> NCHW [n, channels, h*w] (drops zero-padded tail channels)."""
    n, c1, h, w, _ = x.shape
    return from_blocked(x)[:, :channels].reshape(n, channels, h * w)


def softmax(x: torch.Tensor, dim: int, scale: float = 1.0, half_to_float: bool = False) -> torch.Tensor:
    """Attention / generic softmax: an fp16 eager multiply by scale first when
    scale != 1 (whole_blocked.py:101-102), then torch.softmax (verify_softmax.py:67-72)."""
    if scale != 1.0:
        x = x * scale
    if half_to_float:
        return torch.softmax(x.float(), dim)
    return torch.softmax(x, dim)


def make_anchors(shapes: Sequence[Tuple[int, int]], strides: Sequence[float]):
    """fp16 grid-cell centres and strides (whole_blocked.py:124-135)."""
    points, stride_rows = [], []
    for (h, w), s in zip(shapes, strides):
        y, x = torch.meshgrid(torch.arange(h, dtype=torch.float16) + 0.5,
                              torch.arange(w, dtype=torch.float16) + 0.5, indexing="ij")
        points.append(torch.stack((x, y), 0).reshape(2, -1))
        stride_rows.append(torch.full((1, h * w), s, dtype=torch.float16))
    return torch.cat(points, -1), torch.cat(stride_rows, -1)


def dfl(box: torch.Tensor) -> torch.Tensor:
    """Ultralytics DFL(16) in fp16 eager: softmax over the 16 bins of the
    [b, 4, 16, a] view, then the 1x1 conv with arange(16) weights."""
    b, _, a = box.shape
    prob = box.view(b, 4, 16, a).transpose(2, 1).softmax(1)
    weight = torch.arange(16, dtype=box.dtype).view(1, 16, 1, 1)
    return F.conv2d(prob, weight).view(b, 4, a)


def dfl_sequential(box: torch.Tensor) -> torch.Tensor:
    """The DFL expectation in the reference's order, written out: fp16 softmax
    probabilities over the 16 bins (CPU eager), then sum_{i=1..15} p_i * i
    accumulated in FP32 from bin 1 upwards and rounded once to fp16 -- the 1x1
    conv with arange(16) weights of whole_blocked.py:138 (each product p_i * i of
    an fp16 value and a 4-bit integer is exact in FP32, so only the additions
    round).  CPU eager's fp16 conv gives the same bits (tests/test_oracle.py)."""
    b, _, a = box.shape
    prob = box.view(b, 4, 16, a).transpose(2, 1).softmax(1).float()  # [b, 16, 4, a]
    acc = torch.zeros(b, 4, a)
    for i in range(1, 16):
        acc = acc + prob[:, i] * float(i)
    return acc.half()


def decode_from_distances(distance: torch.Tensor, cls: torch.Tensor, shapes, strides,
                          xywh: bool = True) -> torch.Tensor:
    """The decode after the DFL (whole_blocked.py:139-146) on CPU fp16 eager:
    lower = anchors - lt, upper = anchors + rb, xywh ((l+u)/2, u-l) or xyxy,
    times the level stride, then cat with sigmoid(cls)."""
    anchors, stride_row = make_anchors(shapes, strides)
    left_top, right_bottom = distance.split((2, 2), dim=1)
    lower, upper = anchors.unsqueeze(0) - left_top, anchors.unsqueeze(0) + right_bottom
    if xywh:
        boxes = torch.cat(((lower + upper) / 2, upper - lower), 1) * stride_row
    else:
        boxes = torch.cat((lower, upper), 1) * stride_row
    return torch.cat((boxes, cls.sigmoid()), 1)


def dfl_decode(box: torch.Tensor, cls: torch.Tensor, shapes, strides, xywh: bool = True) -> torch.Tensor:
    """anchorfree_predictions (whole_blocked.py:118-146) on CPU fp16 eager."""
    return decode_from_distances(dfl(box), cls, shapes, strides, xywh)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
              prescale: bool = False) -> torch.Tensor:
    """C2PSA Attention core in CPU eager fp16 (attention_forward whole_blocked.py:91-103):
    attn = (q^T @ k) * scale, or with ``prescale`` (attention_scale_before_matmul,
    whole_blocked.py:96-99) attn = (q * scale)^T @ k; attn = softmax(attn, -1);
    out = v @ attn^T.

    q, k [B, h, kd, N], v [B, h, hd, N] fp16; every op rounds to fp16 as the
    reference's separate ATen ops do."""
    if prescale:
        attn = (q * scale).transpose(-2, -1) @ k
    else:
        attn = (q.transpose(-2, -1) @ k) * scale
    attn = attn.softmax(dim=-1)
    return v @ attn.transpose(-2, -1)


def conv_pack_weights(w: torch.Tensor) -> torch.Tensor:
    """OIHW [co, ci, k, k] -> the reference's prepared layout [ceil(ci/16), k*k, co64, 16]
    (blocked_c2f.py:66: reshape(co, ci/16, 16, k*k).permute(1, 3, 0, 2), co padded to 64
    as prepare() does, conv_img.cpp:371-383; ci padded to 16 with zeros)."""
    co, ci, k, _ = w.shape
    cip, cop = (ci + 15) // 16 * 16, (co + 63) // 64 * 64
    full = torch.zeros(cop, cip, k, k, dtype=w.dtype)
    full[:co, :ci] = w
    return full.reshape(cop, cip // 16, 16, k * k).permute(1, 3, 0, 2).contiguous()


def conv2d(x: torch.Tensor, w: torch.Tensor, bias, stride: int, silu: bool) -> torch.Tensor:
    """The reference's fused conv (convolution_native conv_flow.cpp:45-121) on the CPU:
    x NC1HWC0 fp16 [n, c1, h, w, 16] (zero channels past w's ci), w OIHW fp16, bias fp16
    [co] or None; FP32 conv + bias, then s / (1 + exp(-s)) in FP32 when ``silu``, one
    rounding to fp16.  Returns NCHW fp16 [n, co, oh, ow]."""
    xn = from_blocked(x).float()[:, : w.shape[1]]
    k = w.shape[-1]
    s = F.conv2d(xn, w.float(), None if bias is None else bias.float(), stride=stride, padding=(k - 1) // 2)
    if silu:
        s = s / (1.0 + torch.exp(-s))
    return s.half()


def depthwise(x: torch.Tensor, w: torch.Tensor, bias, kernel: int, stride: int, silu: bool) -> torch.Tensor:
    """The reference's depthwise kernel (depthwise_flow.cpp:60-162) on the CPU in its own
    operation order: acc = 0, then for ky, for kx: acc = acc + x * w (FP32 tensors, each
    product and sum rounded), + bias, s / (1 + exp(-s)) when ``silu``, one rounding to fp16.
    x NC1HWC0 fp16 [n, c1, h, w, 16], w [C, 1, k, k] fp16.  Returns NC1HWC0."""
    n, c1, h, wd, _ = x.shape
    pad = kernel // 2
    xp = F.pad(x.float(), (0, 0, pad, pad, pad, pad))  # zero border in W and H
    oh, ow = (h + 2 * pad - kernel) // stride + 1, (wd + 2 * pad - kernel) // stride + 1
    wt = w.float().reshape(c1, 16, kernel, kernel)
    acc = torch.zeros(n, c1, oh, ow, 16)
    for ky in range(kernel):
        for kx in range(kernel):
            src = xp[:, :, ky: ky + (oh - 1) * stride + 1: stride, kx: kx + (ow - 1) * stride + 1: stride, :]
            acc = acc + src * wt[:, :, ky, kx].reshape(1, c1, 1, 1, 16)
    if bias is not None:
        acc = acc + bias.float().reshape(1, c1, 1, 1, 16)
    if silu:
        acc = acc / (1.0 + torch.exp(-acc))
    return acc.half()
