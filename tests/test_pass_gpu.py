"""GPU parity of the whole YOLOv8s-640 non-conv op pass.

Every intermediate (SiLU, residual add, concat, SPPF, upsample, the restored
[B,144,8400] head) must be bit-identical to the CPU-eager pass on the same
inputs; the decoded output is held to the decode tolerance of
test_softmax_gpu.  The CUDA-graph replay must equal eager bitwise."""
from __future__ import annotations

import pytest
import torch

from conftest import assert_bits_equal
from oracle import ops as oops
from oracle import yolo as oyolo
from test_softmax_gpu import _check_decode

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 2])
def test_yolov8s_pass_matches_cpu_eager(device, batch):
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(640)
    inputs = yolo.synthetic_inputs(plan, batch, "cpu", seed=4)
    gpu = yolo.OpPass(plan, {k: v.to(device) for k, v in inputs.items()})
    out = gpu.run()
    want, buffers, head = oyolo.run_pass(plan, inputs, keep=True)
    for step in plan.steps:
        if step.output is not None:
            assert_bits_equal(gpu.buffers[step.output], buffers[step.output], f"{step.op} {step.output}")
    assert_bits_equal(gpu.head, head, "head")
    _check_decode(out, want, plan.levels, plan.strides)


def test_yolov8s_pass_graph_replay_equals_eager(device):
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(640)
    inputs = yolo.synthetic_inputs(plan, 2, device, seed=4)
    p = yolo.OpPass(plan, inputs)
    eager = p.run().clone()
    p.capture()
    for _ in range(3):
        replayed = p.replay()
    torch.cuda.synchronize()
    assert_bits_equal(replayed, eager, "graph replay")


def test_smaller_resolution_pass(device):
    """A 320x320 plan exercises odd-free smaller grids end to end."""
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(320)
    inputs = yolo.synthetic_inputs(plan, 1, "cpu", seed=7)
    gpu = yolo.OpPass(plan, {k: v.to(device) for k, v in inputs.items()})
    out = gpu.run()
    want, buffers, head = oyolo.run_pass(plan, inputs, keep=True)
    assert_bits_equal(gpu.head, head, "head")
    _check_decode(out, want, plan.levels, plan.strides)


@pytest.mark.parametrize("batch", [1, 3])
def test_concat_in_place_equals_op_by_op(device, batch):
    """Zero-copy concat plan: same tensors, no concat kernels."""
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(640)
    inputs = yolo.synthetic_inputs(plan, batch, device, seed=11)
    plain = yolo.OpPass(plan, inputs)
    fused = yolo.OpPass(plan, inputs, concat_in_place=True)
    assert len(fused.elided) == 12 and fused.launches_per_pass() == plain.launches_per_pass() - 12
    plain.run()
    fused.run()
    for step in plan.steps:
        if step.output is not None:
            assert_bits_equal(fused.buffers[step.output], plain.buffers[step.output], step.output)
    assert_bits_equal(fused.output, plain.output, "decoded")
    fused.capture()
    fused.replay()
    torch.cuda.synchronize()
    assert_bits_equal(fused.output, plain.output, "decoded after replay")


@pytest.mark.parametrize("concat_in_place", [False, True])
def test_silu_add_fusion_equals_op_by_op(device, concat_in_place):
    """The six bottleneck SiLUs run inside their residual adds: every tensor the
    fused pass still makes is bit-identical, six fewer launches, 6 x 4 B per element
    of those activations fewer algorithmic bytes; the CPU-eager pass agrees at B=2."""
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(640)
    inputs = yolo.synthetic_inputs(plan, 2, "cpu", seed=12)
    dev = {k: v.to(device) for k, v in inputs.items()}
    plain = yolo.OpPass(plan, dev, concat_in_place=concat_in_place)
    fused = yolo.OpPass(plan, dev, concat_in_place=concat_in_place, fuse_silu_add=True)
    assert len(fused.fused) == 6 and fused.launches_per_pass() == plain.launches_per_pass() - 6
    skipped = {silu.output for _, silu in fused.fused.values()}
    saved = sum(plan.step_bytes(silu) for _, silu in fused.fused.values())
    assert plain.bytes_per_image() - fused.bytes_per_image() == saved
    plain.run()
    fused.run()
    want, buffers, head = oyolo.run_pass(plan, inputs, keep=True)
    for step in plan.steps:
        if step.output is not None and step.output not in skipped:
            assert_bits_equal(fused.buffers[step.output], plain.buffers[step.output], step.output)
            assert_bits_equal(fused.buffers[step.output], buffers[step.output], f"{step.op} {step.output} (CPU)")
    assert_bits_equal(fused.output, plain.output, "decoded")
    assert_bits_equal(fused.head, head, "head (CPU)")
    fused.capture()
    fused.replay()
    torch.cuda.synchronize()
    assert_bits_equal(fused.output, plain.output, "decoded after replay")

