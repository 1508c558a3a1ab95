"""CPU checks of the convolution oracles and the conv list (no GPU).

* The packed-weight layout follows the reference's formula
  packed[cb][tap][o][c] = w[o][16 cb + c][tap] (blocked_c2f.py:66), co padded to 64.
* The depthwise oracle (the reference's own FP32 order) agrees with PyTorch's
  grouped convolution to FP32 rounding.
* The YOLOv8s conv list reproduces the model's published 28.6 GFLOPs at 640.
* The GPU entry points refuse CPU tensors (no CPU fallback)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import ops as oops


def test_conv_pack_weights_formula():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(70, 35, 3, 3, generator=g).half()
    p = oops.conv_pack_weights(w)
    assert tuple(p.shape) == (3, 9, 128, 16)
    for cb in range(3):
        for tap in range(9):
            for o in (0, 5, 69, 70, 127):
                for c in (0, 7, 15):
                    ci = 16 * cb + c
                    want = w[o, ci].reshape(-1)[tap] if o < 70 and ci < 35 else torch.tensor(0.0).half()
                    assert p[cb, tap, o, c] == want


@pytest.mark.parametrize("k,s", [(3, 1), (3, 2), (5, 1), (7, 2), (1, 1)])
def test_depthwise_oracle_matches_grouped_conv(k, s):
    g = torch.Generator().manual_seed(k * 10 + s)
    c, h, w = 32, 19, 23
    x = torch.randn(1, c // 16, h, w, 16, generator=g).half()
    wt = (torch.randn(c, 1, k, k, generator=g) / k).half()
    b = (torch.randn(c, generator=g) * 0.1).half()
    got = oops.from_blocked(oops.depthwise(x, wt, b, k, s, False)).float()
    want = F.conv2d(oops.from_blocked(x).float(), wt.float(), b.float(), stride=s, padding=k // 2, groups=c)
    assert torch.allclose(got, want.half().float(), atol=2e-3, rtol=2 ** -9)


def test_conv2d_oracle_matches_plain_conv():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, 3, 16, 16, generator=g).half()
    w = torch.randn(32, 3, 6, 6, generator=g).half()
    got = oops.from_blocked(oops.pack_padded(oops.conv2d(oops.pack_padded(x), w, None, 2, False).float()))
    want = F.conv2d(x.float(), w.float(), None, stride=2, padding=2)
    assert torch.allclose(got.float()[:, :32], want.half().float(), atol=1e-2, rtol=2 ** -9)


def test_yolov8s_conv_list():
    from thintnpu_b200 import yolo
    convs = yolo.yolov8s_convs(640)
    assert len(convs) == 63 and sum(c.act for c in convs) == 57
    assert abs(sum(c.flops for c in convs) / 1e9 - 28.6) < 0.05  # the model's published GFLOPs
    plan = yolo.yolov8s_plan(640)
    # every activated conv output of the op pass has a conv here with the same shape
    outs = sorted((c.cout, c.out_hw) for c in convs)
    assert len(plan.conv_inputs) == 63 and len(outs) == 63


def test_gpu_entry_points_refuse_cpu_tensors():
    import thintnpu_b200 as ttn
    x = torch.zeros(1, 2, 8, 8, 16, dtype=torch.float16)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        ttn.conv2d(x, torch.zeros(2, 9, 64, 16, dtype=torch.float16), None, 64, 3, 1)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        ttn.depthwise(x, torch.zeros(2, 3, 3, 16, dtype=torch.float16), None, 3, 1)
    q = torch.zeros(1, 1, 32, 64, dtype=torch.float16)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        ttn.attention(q, q, torch.zeros(1, 1, 64, 64, dtype=torch.float16), 1.0)


def _c2f_parts(c_in=64, c=32, n=1, c_out=64, k_cv1=1, k_m=3, cv2_in=None):
    conv = lambda co, ci, k: (torch.zeros(co, ci, k, k, dtype=torch.float16), torch.zeros(co, dtype=torch.float16))
    return (conv(2 * c, c_in, k_cv1), [(conv(c, c, k_m), conv(c, c, k_m)) for _ in range(n)],
            conv(c_out, (2 + n) * c if cv2_in is None else cv2_in, 1))


@pytest.mark.parametrize("kwargs,match", [
    (dict(k_cv1=3), "cv1 must be 1x1"),
    (dict(c=24), "cv1 must be 1x1 with 2c outputs"),
    (dict(cv2_in=64), "cv2 must be 1x1 from"),
    (dict(c_out=40), "c_out % 16"),
    (dict(k_m=1), "bottleneck convs must be 3x3"),
])
def test_c2f_region_checks_its_weights(kwargs, match):
    """The region (blocked_c2f.py:28-68 checks the module's exact shapes) refuses
    malformed weights before any GPU work."""
    from thintnpu_b200.yolo import C2fRegion
    with pytest.raises(RuntimeError, match=match):
        C2fRegion(*_c2f_parts(**kwargs))


def test_c2f_region_needs_cuda_weights():
    from thintnpu_b200.yolo import C2fRegion
    with pytest.raises(RuntimeError, match="CUDA"):
        C2fRegion(*_c2f_parts())
