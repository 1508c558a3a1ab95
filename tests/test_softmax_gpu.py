"""GPU parity: softmax (rows, strided dims, DFL view, attention with scale) and
the fused Detect decode vs PyTorch CPU eager.

Tolerances: softmax within 1e-3 (absolute on fp16 probabilities, the
reference's verify_softmax.py gate, which also bounds the north star's 1e-3
relative on the dominant entries); non-finite positions must match exactly.
Decode: checked in its two halves -- the DFL distances within 1 fp16 ulp of the
reference-order restatement and everything after them bit-exact
(check_decode_trace) -- and end to end against the CPU-eager chain: scores
bit-exact, boxes within the bound _check_decode derives from a 1-ulp distance
flip."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import assert_bits_equal, ulp16, ulp_diff
from oracle import ops as oops

pytestmark = pytest.mark.gpu


def compare(got: torch.Tensor, want: torch.Tensor, tol: float) -> float:
    got = got.cpu()
    assert got.dtype == want.dtype and got.shape == want.shape
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    assert torch.equal(torch.isposinf(got), torch.isposinf(want))
    assert torch.equal(torch.isneginf(got), torch.isneginf(want))
    finite = torch.isfinite(want)
    err = (got.float()[finite] - want.float()[finite]).abs().max().item() if finite.any() else 0.0
    assert err <= tol, err
    return err


SHAPES = [((), (0, -1)), ((0,), (0,)), ((2, 0, 3), (0, 1, 2)), ((1,), (0,)), ((3,), (0,)),
          ((7,), (-1,)), ((100,), (0,)), ((3, 16), (-1, 0)), ((5, 1000), (1,)), ((2, 2049), (1,)),
          ((2, 4097), (-1,)), ((2, 65537), (-1,)), ((2, 3, 7), (0, 1, 2, -2)), ((2, 16, 17), (1,)),
          ((2, 1000, 17), (1,)), ((3, 7, 1), (1,)), ((1, 4, 16, 8400), (1, 2)),
          ((1, 16, 4, 8400), (1,)), ((2, 4, 16, 2100), (2,)), ((64, 400), (-1,)), ((3, 800), (-1,))]


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape,dims", SHAPES)
def test_softmax_shapes(device, dtype, shape, dims):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(2718)
    cpu = (torch.randn(shape, generator=g) * 3).to(dtype)
    tol = 1e-3 if dtype == torch.float16 else 1e-5
    for dim in dims:
        compare(ttn.softmax(cpu.to(device), dim), torch.softmax(cpu, dim), tol)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_softmax_views_shifts_nonfinite(device, dtype):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(2718)
    tol = 1e-3 if dtype == torch.float16 else 1e-5
    for shape, dim in (((3, 1000), -1), ((2, 16, 37), 1), ((2, 1000, 17), 1)):
        for shift in (-10000, 10000):
            cpu = (torch.randn(shape, generator=g) * 10 + shift).to(dtype)
            compare(ttn.softmax(cpu.to(device), dim), torch.softmax(cpu, dim), tol)
        cpu = torch.zeros(shape, dtype=dtype)
        compare(ttn.softmax(cpu.to(device), dim), torch.softmax(cpu, dim), tol)
    cpu = torch.randn(2, 3, 7, generator=g).to(dtype)
    dev = cpu.to(device)
    for dim in (0, 1, -1):
        compare(ttn.softmax(dev.transpose(0, 2), dim), torch.softmax(cpu.transpose(0, 2), dim), tol)
    compare(ttn.softmax(dev.as_strided((2, 3, 5), (21, 7, 1), 1), -1), torch.softmax(cpu[:, :, 1:6], -1), tol)
    compare(ttn.softmax(dev.as_strided((2, 3, 5), (21, 7, 1), 1), 1), torch.softmax(cpu[:, :, 1:6], 1), tol)
    compare(ttn.softmax(dev.unsqueeze(0).expand(4, -1, -1, -1), 0),
            torch.softmax(cpu.unsqueeze(0).expand(4, -1, -1, -1), 0), tol)
    for values in ([float("-inf"), 0, 1], [float("-inf")] * 3, [0, float("inf"), 1], [0, float("nan"), 1]):
        a = torch.tensor(values, dtype=dtype)
        for shape, dim in (((1, 3), 1), ((3, 1), 0), ((3, 17), 0)):
            cpu = a.reshape((1, 3) if dim else (3, 1)).expand(shape).contiguous()
            compare(ttn.softmax(cpu.to(device), dim), torch.softmax(cpu, dim), tol)
    mixed = torch.tensor([[0, 0, float("-inf"), 0, 0], [1, float("nan"), float("-inf"), float("inf"), float("-inf")],
                          [2, 2, float("-inf"), 1, 3]], dtype=dtype)
    compare(ttn.softmax(mixed.to(device), 0), torch.softmax(mixed, 0), tol)
    compare(ttn.softmax(mixed.t().contiguous().to(device), 1), torch.softmax(mixed.t().contiguous(), 1), tol)


def test_softmax_half_to_float(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(5)
    for shape, dim in (((3, 1000), -1), ((2, 16, 17), 1)):
        cpu = torch.randn(shape, generator=g).half()
        compare(ttn.softmax(cpu.to(device), dim, half_to_float=True), torch.softmax(cpu.float(), dim), 1e-5)


@pytest.mark.parametrize("width", [16, 80, 1040, 8400])
def test_dfl_softmax_view(device, width):
    """aten::_softmax over the [b,16,4,a] transposed DFL view (verify_dfl_softmax.py)."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(1928)
    cpu = (torch.randn(2, 4, 16, width, generator=g) * 3).half()
    view = lambda t: t.transpose(1, 2)
    compare(ttn.softmax(view(cpu.to(device)), 1), torch.softmax(view(cpu), 1), 1e-3)
    special = cpu.clone()
    special[:, :, 5, 3] = float("nan")
    special[:, 1, :, 7] = float("-inf")
    compare(ttn.softmax(view(special.to(device)), 1), torch.softmax(view(special), 1), 1e-3)


@pytest.mark.parametrize("batch", [1, 4])
def test_config3_attention_softmax_with_scale(device, batch):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(3)
    scores = torch.randn(batch, 4, 400, 400, generator=g).half()
    scale = 32 ** -0.5
    got = ttn.softmax(scores.to(device), -1, scale=scale)
    want = oops.softmax(scores, -1, scale=scale)
    err = compare(got, want, 1e-3)
    # relative error on probabilities above 1e-3
    big = want.float() > 1e-3
    rel = ((got.cpu().float() - want.float()).abs() / want.float())[big].max().item()
    assert rel <= 1e-3 + 2 ** -10, (err, rel)


def _decode_inputs(batch, seed=2, nc=80, shapes=((80, 80), (40, 40), (20, 20))):
    g = torch.Generator().manual_seed(seed)
    a = sum(h * w for h, w in shapes)
    box = (torch.randn(batch, 64, a, generator=g) * 2).half()
    cls = (torch.randn(batch, nc, a, generator=g) * 3).half()
    return box, cls, list(shapes)


def _check_decode(got, want, shapes, strides):
    """Decode output vs the CPU-eager chain: scores bit-exact; every box value within
    stride * (2 ulp16(|anchor| + 16) + 2^-6) + 2 ulp16(box).  The one non-exact step
    is an fp16 rounding flip of a DFL probability, which moves a distance d (< 16)
    by at most one ulp (2^-7; check_decode_trace pins that and the exactness of
    the rest); anchor -+ d then moves by up to one fp16 step at its magnitude
    (|anchor| + 16), (l + u) / 2 and u - l by two, and the stride scales it.
    Returns the bit-equal fraction of the box values."""
    got = got.cpu()
    assert_bits_equal(got[:, 4:], want[:, 4:], "scores")
    points, stride_row = oops.make_anchors(shapes, strides)
    step = ulp16(points.float().abs().max(0).values + 16)
    err = (got[:, :4].float() - want[:, :4].float()).abs()
    bound = stride_row.float() * (2 * step + 2.0 ** -6) + 2 * ulp16(want[:, :4])
    assert torch.all(err <= bound), (err - bound).max()
    return float((got[:, :4].view(torch.int16) == want[:, :4].view(torch.int16)).float().mean())


@pytest.mark.parametrize("xywh", [True, False])
def test_config2_dfl_decode(device, xywh):
    import thintnpu_b200 as ttn
    box, cls, shapes = _decode_inputs(1)
    strides = [8.0, 16.0, 32.0]
    got = ttn.dfl_decode(box.to(device), cls.to(device), shapes, strides, xywh=xywh)
    want = oops.dfl_decode(box, cls, shapes, strides, xywh=xywh)
    exact = _check_decode(got, want, shapes, strides)
    assert exact > 0.98, exact


def test_dfl_decode_views_batches_and_odd_grids(device):
    import thintnpu_b200 as ttn
    # [B, 144, A] head split into box/cls views, batch 3, unaligned odd grid
    g = torch.Generator().manual_seed(11)
    shapes = [(13, 17), (7, 9), (3, 5)]
    a = sum(h * w for h, w in shapes)
    head = (torch.randn(3, 64 + 17, a, generator=g) * 2).half()
    strides = [8.0, 16.0, 32.0]
    dev = head.to(device)
    got = ttn.dfl_decode(dev[:, :64], dev[:, 64:], shapes, strides)
    want = oops.dfl_decode(head[:, :64].contiguous(), head[:, 64:].contiguous(), shapes, strides)
    _check_decode(got, want, shapes, strides)


@pytest.mark.parametrize("batch,nc", [(52, 80), (2, 120)])
def test_dfl_decode_head_views_tiled(device, batch, nc):
    """Box and class rows as views of one [B, 64 + nc, 8400] head: the tiled box
    kernel plus the row-family sigmoid (table kernel at B=52, arithmetic at B=2)."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(5 + nc)
    shapes = [(80, 80), (40, 40), (20, 20)]
    head = (torch.randn(batch, 64 + nc, 8400, generator=g) * 3).half()
    strides = [8.0, 16.0, 32.0]
    dev = head.to(device)
    got = ttn.dfl_decode(dev[:, :64], dev[:, 64:], shapes, strides)
    want = oops.dfl_decode(head[:, :64].contiguous(), head[:, 64:].contiguous(), shapes, strides)
    exact = _check_decode(got, want, shapes, strides)
    assert exact > 0.98, exact


def check_decode_trace(box, cls, shapes, strides, xywh, device):
    """The decode checked in its two halves (box, cls: CPU fp16 logits):

    * the DFL distances the GPU decoded from (the trace entry point) within 1 fp16
      ulp of the reference-order restatement (oracle.dfl_sequential; CPU eager's
      conv gives the same bits) and at least 95% bit-equal -- the only
      difference left is an fp16 rounding flip of a probability, where the two
      exps differ in the last bits (CPU eager's own exp differs between the
      vector body and the scalar tail of its softmax loop, so the bit-equal
      share depends on the grid: >= 99.5% at 8400 anchors, 97% on a 54-anchor
      grid);
    * everything after the DFL bit-exact: CPU eager's anchor arithmetic and
      sigmoid applied to the GPU's own distances equals the GPU output.
    Returns the bit-equal fraction of the distances."""
    import thintnpu_b200 as ttn
    n, _, a = box.shape
    dist = torch.empty(n, 4, a, dtype=torch.float16, device=device)
    got = ttn.dfl_decode(box.to(device), cls.to(device), shapes, strides, xywh=xywh, distances=dist)
    d = ulp_diff(dist, oops.dfl_sequential(box))
    assert d.max() <= 1, d.max()
    exact = float((d == 0).mean())
    assert exact >= 0.95, exact
    again = oops.decode_from_distances(dist.cpu(), cls, shapes, strides, xywh)
    assert_bits_equal(got, again, "decode of the GPU's own distances")
    return exact


@pytest.mark.parametrize("xywh", [True, False])
@pytest.mark.parametrize("grid", ["v8-640", "odd", "even"])
def test_decode_halves_exact(device, xywh, grid):
    """Tiled (anchors % 8 == 0), paired (even) and single-anchor kernels."""
    shapes = {"v8-640": [(80, 80), (40, 40), (20, 20)], "odd": [(13, 17), (7, 9), (3, 5)],
              "even": [(6, 7), (3, 4)]}[grid]
    box, cls, shapes = _decode_inputs(3, seed=41, shapes=tuple(shapes))
    check_decode_trace(box, cls, shapes, [8.0, 16.0, 32.0][:len(shapes)], xywh, device)


def test_decode_trace_special_rows(device):
    """verify_dfl_softmax.py's special rows (NaN, -inf, zeros, large shift) through
    the traced decode."""
    box, cls, shapes = _decode_inputs(2, seed=43)
    box[0, 5, 7] = float("nan")
    box[1, 16:32, 9] = float("-inf")
    box[1, 32:48, 11] = 0
    box[0, :, 13] = 6000
    import thintnpu_b200 as ttn
    n, _, a = box.shape
    dist = torch.empty(n, 4, a, dtype=torch.float16, device=device)
    got = ttn.dfl_decode(box.to(device), cls.to(device), shapes, [8.0, 16.0, 32.0], distances=dist)
    want = oops.dfl_sequential(box)
    assert torch.equal(torch.isnan(dist.cpu()), torch.isnan(want))
    again = oops.decode_from_distances(dist.cpu(), cls, shapes, [8.0, 16.0, 32.0])
    assert_bits_equal(got, again, "decode of the GPU's own distances")
