"""The YOLOv8s op pass on CPU eager (test infrastructure and CPU baseline only).

Walks the same Plan as thintnpu_b200.yolo.OpPass, one PyTorch CPU op per step:
F.silu, fp16 add, torch.cat, F.max_pool2d (FP32, as verify_flow_ops.py:25-27),
F.interpolate nearest, the NC1HWC0 -> NCHW permute, and the Ultralytics decode
chain of whole_blocked.py:118-146.
"""
from __future__ import annotations

from typing import Dict

import torch

from . import ops as oops


def _run_step(plan, step, buffers, head):
    """One op-pass step on CPU eager; returns the decoded tensor for the decode step."""
    def view(ref):
        t = buffers[ref.name]
        return t[:, ref.start:ref.start + ref.count]

    if step.op == "silu":
        buffers[step.output] = oops.silu(view(step.inputs[0]))
    elif step.op == "add":
        buffers[step.output] = view(step.inputs[0]) + view(step.inputs[1])
    elif step.op == "cat":
        buffers[step.output] = torch.cat([view(r) for r in step.inputs], 1)
    elif step.op == "sppf":
        buffers[step.output] = oops.sppf(view(step.inputs[0]).contiguous(), step.attrs[0])
    elif step.op == "upsample":
        buffers[step.output] = oops.upsample_blocked(view(step.inputs[0]).contiguous())
    elif step.op == "restore":
        channel0, channels, anchor0 = step.attrs
        x = view(step.inputs[0])
        hw = x.size(2) * x.size(3)
        head[:, channel0:channel0 + channels, anchor0:anchor0 + hw] = oops.unpack(x, channels)
    elif step.op == "decode":
        return oops.dfl_decode(head[:, :64], head[:, 64:], plan.levels, plan.strides, xywh=step.attrs[0])
    return None


def run_pass(plan, inputs: Dict[str, torch.Tensor], keep: bool = False, fused_act: bool = False):
    """inputs: conv name -> CPU fp16 [B, c1, h, w, 16].  Returns the decoded
    [B, 4+nc, anchors] tensor, and with ``keep`` also every step output.

    With ``fused_act`` the inputs are the activated conv outputs, keyed by the SiLU
    steps' output names (and the raw names for the convs without activation), and
    the SiLU steps are skipped: the op pass of a model whose convs fuse the SiLU."""
    buffers = dict(inputs)
    batch = next(iter(inputs.values())).size(0)
    head = torch.zeros((batch, 64 + plan.nc, plan.anchors), dtype=torch.float16)
    out = None
    for step in plan.steps:
        if fused_act and step.op == "silu":
            continue
        got = _run_step(plan, step, buffers, head)
        if got is not None:
            out = got
    if keep:
        return out, buffers, head
    return out


def run_model(plan, weights, image: torch.Tensor, keep: bool = False):
    """The whole model on CPU eager in model order (plan.order): every conv is the
    reference's fused conv (oracle.ops.conv2d: FP32 conv + bias, FP32 SiLU when the
    conv is activated, one fp16 rounding) on its source buffer (the image for the
    stem), every other step as in run_pass.  weights: (OIHW fp16, bias fp16) per conv;
    image: NC1HWC0 [B, 1, S, S, 16] fp16.  Returns the decoded tensor (and with
    ``keep`` every buffer and the head)."""
    act_of = {st.inputs[0].name: st.output for st in plan.steps if st.op == "silu"}
    buffers: Dict[str, torch.Tensor] = {}
    head = torch.zeros((image.size(0), 64 + plan.nc, plan.anchors), dtype=torch.float16)
    out = None
    for kind, index in plan.order:
        if kind == "conv":
            name = plan.conv_inputs[index]
            src = plan.conv_sources[index]
            x = image if src is None else buffers[src.name][:, src.start:src.start + src.count]
            w, b = weights[index]
            _, stride = plan.conv_kernels[index]
            y = oops.conv2d(x.contiguous(), w.cpu(), b.cpu(), stride, name in act_of)
            buffers[act_of.get(name, name)] = oops.to_blocked(y)
        else:
            step = plan.steps[index]
            if step.op == "silu":
                continue
            got = _run_step(plan, step, buffers, head)
            if got is not None:
                out = got
    if keep:
        return out, buffers, head
    return out
