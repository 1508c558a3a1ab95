"""The whole-model plan on the CPU: every conv's recorded input and kernel agree
with the YOLOv8s conv list, the model order puts each conv after the step that
makes its input, and the CPU chain (oracle.yolo.run_model) equals its own op pass
run on its conv outputs."""
from __future__ import annotations

import pytest
import torch

from oracle import yolo as oyolo
from thintnpu_b200 import yolo


@pytest.mark.parametrize("imgsz", [320, 640])
def test_conv_wiring_matches_the_conv_list(imgsz):
    plan = yolo.yolov8s_plan(imgsz)
    specs = yolo.yolov8s_convs(imgsz)
    assert len(plan.conv_inputs) == len(plan.conv_sources) == len(plan.conv_kernels) == len(specs) == 63
    for name, src, (k, s), sp in zip(plan.conv_inputs, plan.conv_sources, plan.conv_kernels, specs):
        c1, h, w = plan.shapes[name]
        cin = 3 if src is None else src.count * 16
        in_hw = plan.imgsz if src is None else plan.shapes[src.name][1]
        assert (cin, c1 * 16, k, s, in_hw) == (sp.cin, sp.cout, sp.k, sp.s, sp.h), name
        assert (h, w) == sp.out_hw, name


def test_model_order_is_topological():
    plan = yolo.yolov8s_plan(320)
    made = set()
    act_of = {st.inputs[0].name: st.output for st in plan.steps if st.op == "silu"}
    assert sorted(i for kind, i in plan.order if kind == "conv") == list(range(63))
    assert sorted(i for kind, i in plan.order if kind == "step") == list(range(len(plan.steps)))
    for kind, index in plan.order:
        if kind == "conv":
            src = plan.conv_sources[index]
            assert src is None or src.name in made, (index, src)
            made.add(plan.conv_inputs[index])
        else:
            step = plan.steps[index]
            for ref in step.inputs:
                assert ref.name in made, (step.op, ref)
            if step.output is not None:
                made.add(step.output)
    assert set(act_of.values()) <= made


def test_cpu_chain_equals_its_op_pass():
    plan = yolo.yolov8s_plan(64)
    weights = yolo.model_weights(plan, "cpu")
    image = yolo.synthetic_image(plan, 2, "cpu")
    out, buffers, head = oyolo.run_model(plan, weights, image, keep=True)
    act_of = {st.inputs[0].name: st.output for st in plan.steps if st.op == "silu"}
    inputs = {act_of.get(n, n): buffers[act_of.get(n, n)] for n in plan.conv_inputs}
    again, _, head2 = oyolo.run_pass(plan, inputs, keep=True, fused_act=True)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))
    assert torch.equal(head.view(torch.int16), head2.view(torch.int16))
    assert torch.isfinite(out.float()).all()


def test_conv_launch_count():
    """The stem-shaped conv (one input channel block, 3x3 stride 2, <= 64 outputs)
    launches the tensor-core and the CUDA-core stem kernels; every other conv one."""
    specs = yolo.yolov8s_convs(640)
    assert [sp.launches for sp in specs].count(2) == 1 and specs[0].launches == 2
    assert sum(sp.launches for sp in specs) == 64
    assert yolo.conv_launches(16, 64, 3, 2) == 2 and yolo.conv_launches(32, 64, 3, 2) == 1
    assert yolo.conv_launches(3, 80, 3, 2) == 1 and yolo.conv_launches(3, 32, 1, 1) == 1
