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


def run_pass(plan, inputs: Dict[str, torch.Tensor], keep: bool = False):
    """inputs: conv name -> CPU fp16 [B, c1, h, w, 16].  Returns the decoded
    [B, 4+nc, anchors] tensor, and with ``keep`` also every step output."""
    buffers = dict(inputs)
    batch = next(iter(inputs.values())).size(0)
    head = torch.zeros((batch, 64 + plan.nc, plan.anchors), dtype=torch.float16)

    def view(ref):
        t = buffers[ref.name]
        return t[:, ref.start:ref.start + ref.count]

    out = None
    for step in plan.steps:
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
            out = oops.dfl_decode(head[:, :64], head[:, 64:], plan.levels, plan.strides,
                                  xywh=step.attrs[0])
    if keep:
        return out, buffers, head
    return out
