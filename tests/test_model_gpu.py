"""GPU parity of the whole-model chain (yolo.ModelPass: the 63 tcgen05 convs with
bias + SiLU fused, chained with the op pass in model order, one CUDA graph).

* layer by layer at 320 (B=2): every conv's output, computed on the GPU from the
  GPU's own input buffer, within the conv gate of test_conv_gpu (one fp16 step plus
  the FP32 accumulation-order term, >= 99.5% - 5e-6 K bit-equal) against the
  reference's fused conv on the CPU; every other step's output bit-exact against CPU
  eager run on the GPU's conv outputs; the decode within the decode gate;
* the graph replay and the plain (non zero-copy) schedule bit-identical to the eager
  zero-copy run;
* end to end at 320 (B=1) against the CPU chain from the same image and weights:
  the per-layer rounding differences propagate through 63 convs, so the gate is on
  the decoded scores and boxes (absolute, in probability and pixels; measured on a
  B200: 4.9e-4 and 0.5 px).
"""
from __future__ import annotations

import pytest
import torch

from oracle import ops as oops
from oracle import yolo as oyolo
from test_conv_gpu import _check as conv_gate
from test_softmax_gpu import _check_decode

pytestmark = pytest.mark.gpu


def _model(imgsz, batch, device, concat_in_place=True):
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(imgsz)
    weights = yolo.model_weights(plan, device)
    image = yolo.synthetic_image(plan, batch, device)
    return plan, weights, image, yolo.ModelPass(plan, weights, image, concat_in_place=concat_in_place)


def test_model_layer_by_layer(device):
    import thintnpu_b200 as ttn
    plan, weights, image, model = _model(320, 2, device)
    out = model.run()
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    for index, (src, _, _, cout, k, stride, silu, name) in enumerate(model.convs):
        x = model.conv_input(index).cpu()
        cin = 3 if src is None else src.count * 16
        w, b = weights[index]
        conv_gate(oops.from_blocked(model.buffers[name].cpu()), oops.from_blocked(x)[:, :cin], w.cpu(), b.cpu(),
                  stride, silu)
    inputs = {conv[-1]: model.buffers[conv[-1]].cpu() for conv in model.convs}
    want, buffers, head = oyolo.run_pass(plan, inputs, keep=True, fused_act=True)
    for step in plan.steps:
        if step.output is not None and step.op != "silu":
            got = model.buffers[step.output].cpu()
            assert torch.equal(got.view(torch.int16), buffers[step.output].view(torch.int16)), \
                f"{step.op} {step.output}"
    assert torch.equal(model.head.cpu().view(torch.int16), head.view(torch.int16))
    _check_decode(out, want, plan.levels, plan.strides)


def test_model_graph_and_plain_schedule_match_eager(device):
    _, _, _, model = _model(320, 2, device)
    eager = model.run().clone()
    model.capture(warmup=1)
    replayed = model.replay()
    torch.cuda.synchronize()
    assert torch.equal(replayed.view(torch.int16), eager.view(torch.int16))
    _, _, _, plain = _model(320, 2, device, concat_in_place=False)
    assert torch.equal(plain.run().view(torch.int16), eager.view(torch.int16))
    assert plain.launches_per_pass() - model.launches_per_pass() == len(model.elided)


def test_model_end_to_end_against_cpu_chain(device):
    plan, weights, image, model = _model(320, 1, device)
    got = model.run().cpu().float()
    want = oyolo.run_model(plan, [(w.cpu(), b.cpu()) for w, b in weights], image.cpu()).float()
    score_err = (got[:, 4:] - want[:, 4:]).abs().max().item()
    box_err = (got[:, :4] - want[:, :4]).abs().max().item()
    print(f"end to end at 320: max score error {score_err:.3g}, max box error {box_err:.3g} px")
    assert score_err <= 4e-3, score_err
    assert box_err <= 2.0, box_err
