"""GPU parity at the configurations bench.py times, on the bench's own objects.

``bench.py`` times config 4 at 256 images per GPU (the zero-copy plan, plain
pass as a variant), config 3 at B=64 and config 5 at N=512, and ``--config N``
times configs 1 and 2 at B=256.  These tests build the same objects with the
same seeds (rank 0's), run the same calls, and hold every result to the parity
gate of its row:

* config 5 (N=512, K=300 both modes and both NaN orders; K=511/512/513
  class-aware, both NaN orders): the packed [N, K, 6] rows bit-exact against the
  selection oracle run on CPU-eager fp16 sigmoid bits of the same logits;
* config 3 (B=64): within 1e-3 absolute and 1e-3 relative on probabilities above
  1e-3; non-finite positions exact;
* config 4 (B=256: the timed zero-copy pass with the bottleneck SiLUs fused into
  their adds, the zero-copy pass unfused, and the plain pass): images 0, 128 and
  255 of every step output it makes and of the restored head bit-exact against the
  CPU-eager pass run on those three images alone (images never interact), the
  decode within the decode gate;
* config 1 (B=256): within 2 fp16 ulp of CPU eager plus the FP32 evaluation
  error of the SiLU term (conftest.check_bias_silu_residual), >= 99% bit-equal;
* config 2 (B=256): scores bit-exact, boxes within the decode gate, and the
  decode's two halves (DFL distances <= 1 ulp, the rest bit-exact).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench_configs as bc
from conftest import assert_bits_equal, check_bias_silu_residual
from oracle import ops as oops
from oracle import select as osel
from oracle import yolo as oyolo
from test_softmax_gpu import _check_decode, check_decode_trace, compare

pytestmark = pytest.mark.gpu

CONFIG5_CASES = ([(300, agnostic, nan_last) for agnostic in (False, True) for nan_last in (False, True)] +
                 [(k, False, nan_last) for k in (511, 512, 513) for nan_last in (False, True)])


@pytest.fixture(scope="module")
def config5_n512(device):
    """The bench variant's logits (seed 50, rank 0) on the GPU and their CPU-eager
    sigmoid bits [512, 8400, 84] for the oracle, plus a per-NaN-order stage-1 cache."""
    logits = bc.config5_logits(512, 50, device)
    cpu = logits.cpu().transpose(1, 2)
    scores = cpu.clone()
    scores[..., 4:] = torch.sigmoid(scores[..., 4:])
    bits = scores.contiguous().view(torch.int16).numpy().view(np.uint16)
    return logits, bits, {}


@pytest.mark.parametrize("k,agnostic,nan_last", CONFIG5_CASES)
def test_config5_n512_bit_exact(device, config5_n512, k, agnostic, nan_last):
    logits, bits, stage1 = config5_n512
    cfg = bc.Config5(k, agnostic, nan_last)
    cfg.bind(logits)
    cfg.step()
    got = cfg.out.cpu().view(torch.int32).numpy().view(np.uint32)
    if nan_last not in stage1:
        stage1[nan_last] = osel.class_max(bits, nan_last)
    want = osel.select(bits, k, agnostic, nan_last, stage1=stage1[nan_last])["output"]
    if not np.array_equal(got, want):
        bad = np.argwhere((got != want).any(-1))
        raise AssertionError(f"{len(bad)} rows differ, first at image/rank {bad[0].tolist()}")


def test_config5_bench_setup_matches_test_input(device):
    """The bench variant's own setup (measure_config: seed 50 + rank) builds the
    logits the N=512 tests check."""
    cfg = bc.Config5()
    cfg.setup(512, device, seed=50)
    assert torch.equal(cfg.base.view(torch.int16), bc.config5_logits(512, 50, device).view(torch.int16))
    assert cfg.decoded.stride() == (84 * 8400, 1, 8400)


def test_config3_b64(device):
    cfg = bc.Config3()
    cfg.setup(64, device, seed=30)  # the bench variant's seed at rank 0
    cfg.step()
    x = cfg.x.cpu()
    want = oops.softmax(x, -1, scale=cfg.scale)
    got = cfg.y.cpu()
    compare(got, want, 1e-3)
    big = want.float() > 1e-3
    rel = ((got.float() - want.float()).abs() / want.float())[big].max().item()
    assert rel <= 1e-3 + 2 ** -10, rel


@pytest.mark.parametrize("concat_in_place,fuse", [(True, True), (True, False), (False, False)])
def test_config4_b256_image_slices(device, concat_in_place, fuse):
    """(True, True) is the bench's timed pass; the other two are its variants."""
    from thintnpu_b200 import yolo
    plan = yolo.yolov8s_plan(640)
    inputs = yolo.synthetic_inputs(plan, 256, device, seed=4)  # bench rank 0
    gpu = yolo.OpPass(plan, inputs, concat_in_place=concat_in_place, fuse_silu_add=fuse)
    gpu.capture(warmup=1)
    out = gpu.replay()
    torch.cuda.synchronize()
    images = [0, 128, 255]
    cpu_inputs = {k: v[images].cpu() for k, v in inputs.items()}
    want, buffers, head = oyolo.run_pass(plan, cpu_inputs, keep=True)
    skipped = {silu.output for _, silu in gpu.fused.values()}
    for step in plan.steps:
        if step.output is not None and step.output not in skipped:
            assert_bits_equal(gpu.buffers[step.output][images], buffers[step.output], f"{step.op} {step.output}")
    assert_bits_equal(gpu.head[images], head, "head")
    _check_decode(out[images], want, plan.levels, plan.strides)


def test_config1_b256(device):
    cfg = bc.Config1()
    cfg.setup(256, device, seed=10)  # bench.py --config 1, rank 0
    cfg.step()
    x, b, r = cfg.x.cpu(), cfg.b.cpu(), cfg.r.cpu()
    check_bias_silu_residual(cfg.y, x, b, r, oops.bias_silu_residual(x, b, r))


def test_config2_b256(device):
    cfg = bc.Config2()
    cfg.setup(256, device, seed=20)  # bench.py --config 2, rank 0
    cfg.step()
    want = oops.dfl_decode(cfg.box.cpu(), cfg.cls.cpu(), cfg.shapes, cfg.strides)
    exact = _check_decode(cfg.out, want, cfg.shapes, cfg.strides)
    assert exact > 0.98, exact
    check_decode_trace(cfg.box.cpu(), cfg.cls.cpu(), cfg.shapes, cfg.strides, True, device)
