"""GPU parity (bitwise): concat/split, strided copy, NC1HWC0<->NCHW, upsample,
max-pool and SPPF against the reference tests' CPU formulas (tolerance 0)."""
from __future__ import annotations

import pytest
import torch

from conftest import assert_bits_equal
from oracle import ops as oops

pytestmark = pytest.mark.gpu

SPECIAL = torch.tensor([0., -0., float("nan"), float("inf"), -float("inf")])


def _special(t: torch.Tensor) -> torch.Tensor:
    t = t.clone()
    t.view(-1)[:SPECIAL.numel()] = SPECIAL.to(t.dtype)
    return t


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_cat_dims_and_views(device, dtype):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(42)
    for dim in range(4):
        for outer in (1, 3):
            shape = [outer, 3, 32, 32]
            inputs = []
            for size in (1, 2, 5):
                cur = shape.copy()
                cur[dim] = size if dim != 3 else size * 32
                inputs.append(torch.randn(cur, generator=g).to(dtype))
            assert_bits_equal(ttn.cat([t.to(device) for t in inputs], dim), torch.cat(inputs, dim))
    for length in (16, 8192, 16384 + 16, 131072 + 16):
        inputs = [torch.randn(3, length, generator=g).to(dtype) for _ in range(3)]
        assert_bits_equal(ttn.cat([t.to(device) for t in inputs], -1), torch.cat(inputs, -1))
    for offset in (1, 16):
        src = torch.randn(3 * 64 * 64 + offset, generator=g).to(dtype)
        dev = src.to(device)
        cv, dv = src[offset:].view(3, 64, 64), dev[offset:].view(3, 64, 64)
        assert_bits_equal(ttn.cat([dv] * 2, 1), torch.cat([cv] * 2, 1))
        assert_bits_equal(ttn.cat([dv.transpose(0, 2)] * 2, 1), torch.cat([cv.transpose(0, 2)] * 2, 1))
    src = torch.randn(3, 64, 32, generator=g).to(dtype)
    dev = src.to(device)
    assert_bits_equal(ttn.cat(dev.split(32, 1), 1), torch.cat(src.split(32, 1), 1))
    assert_bits_equal(ttn.cat([dev[:1].expand(3, -1, -1)] * 2, 1), torch.cat([src[:1].expand(3, -1, -1)] * 2, 1))
    empty = torch.empty(0, dtype=dtype)
    assert_bits_equal(ttn.cat([empty.to(device), dev, empty.to(device)], 1), src)
    assert ttn.cat([empty.to(device), empty.to(device)], 0).numel() == 0
    assert_bits_equal(ttn.cat([torch.empty(3, 0, 32, dtype=dtype, device=device), dev], 1), src)
    values = _special(torch.tensor([1.0, -1.0, 0.5] * 40)).to(dtype)
    assert_bits_equal(ttn.cat([values.to(device)] * 2, 0), torch.cat([values] * 2, 0))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_cat_blocked_plan(device, dtype):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(42)
    for count in (1, 2, 3, 4, 6, 8, 9, 17, 70):
        for batch in (1, 3):
            for plane in (20, 80) if count < 20 else (20,):
                cpu = [_special(torch.randn(batch, 1 + i % 3, plane, plane, 16, generator=g).to(dtype))
                       for i in range(count)]
                assert_bits_equal(ttn.cat([v.to(device) for v in cpu], 1), torch.cat(cpu, 1))
    for rows in (8, 81, 129):
        cpu = [torch.randn(1, rows, n, generator=g).to(dtype) for n in (6400, 1600, 400)]
        assert_bits_equal(ttn.cat([v.to(device) for v in cpu], 2), torch.cat(cpu, 2))
    x = torch.randn(3, 12, 40, 40, 16, generator=g).to(dtype)
    for sizes in ((3, 3, 6), (1, 2, 3, 6)):
        assert_bits_equal(ttn.cat(x.to(device).split(sizes, 1), 1), x)


def test_cat_narrow_and_strided_inputs(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(913)
    for rows in (1, 7, 127, 128, 129, 6400):
        for widths in ((2, 2, 12), (1, 7, 24), (3, 5, 8), (6, 10)):
            src = [torch.randn(rows, w, generator=g).half() for w in widths]
            assert_bits_equal(ttn.cat([s.to(device) for s in src], -1), torch.cat(src, -1))
    for transform in (lambda t: t[::3], lambda t: t[:1].expand(273, -1), lambda t: t[:, 1:]):
        src = [torch.randn(273, w + 1, generator=g).half() for w in (2, 2, 12)]
        assert_bits_equal(ttn.cat([transform(s.to(device)) for s in src], -1),
                          torch.cat([transform(s) for s in src], -1))


def test_materialize_views_and_nan_payloads(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(913)
    for dtype in (torch.float16, torch.float32):
        for groups, channels, rows in ((1, 16, 16), (3, 16, 6400), (2, 32, 48), (4, 48, 400),
                                       (2, 7, 19), (1, 85, 96)):
            x = torch.randn(groups, channels, rows, generator=g).to(dtype)
            assert_bits_equal(ttn.contiguous(x.to(device).permute(0, 2, 1)), x.permute(0, 2, 1).contiguous())
        for shape in ((3, 128, 16), (2, 19, 7), (1, 32, 85), (4, 48, 32)):
            x = torch.randn(shape, generator=g).to(dtype)
            for view in (lambda t: t[..., 2:4], lambda t: t[..., 4:], lambda t: t[:, ::2, ::2],
                         lambda t: t[:, :1].expand(-1, 31, -1)):
                assert_bits_equal(ttn.contiguous(view(x.to(device))), view(x).contiguous())
    raw = torch.randint(-32768, 32768, (3, 32, 48), dtype=torch.int16, generator=g).view(torch.float16)
    assert_bits_equal(ttn.contiguous(raw.to(device).transpose(1, 2)), raw.transpose(1, 2).contiguous())
    slices = [raw[..., :2].contiguous(), raw[..., 2:4].contiguous(), raw[..., 4:16].contiguous()]
    assert_bits_equal(ttn.cat([s.to(device) for s in slices], -1), torch.cat(slices, -1))


def test_pack_unpack(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(3)
    for n, c, h, w in ((1, 64, 80, 80), (2, 80, 40, 40), (3, 16, 13, 17), (1, 40, 5, 7), (2, 24, 6, 6),
                       (1, 33, 2, 2)):
        x = torch.randint(-32768, 32768, (n, c, h, w), dtype=torch.int16, generator=g).view(torch.float16)
        packed = ttn.pack(x.to(device))
        assert_bits_equal(packed, oops.pack_padded(x))
        back = ttn.unpack(packed, c)
        assert_bits_equal(back.reshape(n, c, h * w), x.reshape(n, c, h * w))
    # restore straight into a [B, 144, 8400] head at the level's anchor offset
    boxes = [torch.randn(2, 4, s, s, 16, generator=g).half() for s in (80, 40, 20)]
    head = torch.zeros(2, 144, 8400, dtype=torch.float16, device=device)
    offset = 0
    for b in boxes:
        ttn.unpack(b.to(device), 64, out=head[:, :64], out_offset=offset)
        offset += b.size(2) * b.size(3)
    want = torch.cat([oops.unpack(b, 64) for b in boxes], -1)
    assert_bits_equal(head[:, :64], want)
    # odd anchor offset: rows only 2-byte aligned
    odd = torch.zeros(2, 64, 8401, dtype=torch.float16, device=device)
    offset = 1
    for b in boxes:
        ttn.unpack(b.to(device), 64, out=odd, out_offset=offset)
        offset += b.size(2) * b.size(3)
    assert_bits_equal(odd[..., 1:], want)


@pytest.mark.parametrize("c,h,w,k", [(256, 20, 20, 5), (128, 40, 40, 5), (512, 20, 20, 5),
                                     (32, 13, 17, 3), (16, 7, 9, 7), (48, 1, 31, 5), (16, 80, 80, 5)])
def test_maxpool_blocked(device, c, h, w, k):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, c, h, w, generator=g).half()
    xb = oops.to_blocked(x)
    assert_bits_equal(ttn.maxpool_blocked(xb.to(device), k), oops.maxpool_blocked(xb, k))


def test_maxpool_special_values_match_cpu_scan_order(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 32, 9, 11, generator=g).half()
    flat = x.view(-1)
    idx = torch.randperm(flat.numel(), generator=g)
    flat[idx[:60]] = 0.0
    flat[idx[60:120]] = -0.0
    flat[idx[120:140]] = float("inf")
    flat[idx[140:160]] = -float("inf")
    payloads = torch.tensor([0x7E00, 0xFE00, 0x7C01, 0x7D23], dtype=torch.int32).to(torch.int16).view(torch.float16)
    flat[idx[160:168]] = payloads.repeat(2)
    xb = oops.to_blocked(x)
    for k in (3, 5):
        assert_bits_equal(ttn.maxpool_blocked(xb.to(device), k), oops.maxpool_blocked(xb, k), f"k{k}")
        assert_bits_equal(ttn.maxpool2d(x.to(device), k), oops.maxpool_nchw(x, k), f"nchw k{k}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_nchw_pool_and_upsample(device, dtype):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(42)
    for shape in ((1, 2, 5, 7), (2, 3, 13, 11), (1, 64, 80, 80), (1, 64, 40, 40)):
        a = torch.randn(shape, generator=g).to(dtype)
        assert_bits_equal(ttn.maxpool2d(a.to(device)), oops.maxpool_nchw(a, 5))
        assert_bits_equal(ttn.upsample_nearest2d(a.to(device)), oops.upsample_nchw(a))


@pytest.mark.parametrize("c,h,w", [(128, 40, 40), (256, 20, 20), (64, 13, 17), (16, 1, 33)])
def test_upsample_blocked(device, c, h, w):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(0)
    xb = oops.to_blocked(torch.randn(2, c, h, w, generator=g).half())
    assert_bits_equal(ttn.upsample_blocked(xb.to(device)), oops.upsample_blocked(xb))


@pytest.mark.parametrize("n,c1,hw", [(1, 16, 20), (4, 16, 20), (2, 3, 13), (1, 2, 40), (1, 1, 64), (3, 2, 1),
                                     (2, 2, 16), (1, 3, 22)])
def test_sppf(device, n, c1, hw):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(9)
    x = torch.randn(n, c1, hw, hw, 16, generator=g).half()
    assert_bits_equal(ttn.sppf(x.to(device), 5), oops.sppf(x, 5))


@pytest.mark.parametrize("n,c1,h,w", [(2, 3, 13, 7), (1, 2, 5, 22), (1, 1, 1, 9), (2, 1, 3, 1), (1, 2, 21, 18),
                                      (3, 5, 4, 4), (1, 1, 30, 31), (2, 3, 20, 7), (1, 2, 16, 32), (1, 1, 10, 1),
                                      (2, 2, 20, 31), (1, 2, 10, 10), (3, 1, 16, 2)])
def test_sppf_rectangular_planes(device, n, c1, h, w):
    """Rows and columns that are not multiples of the kernel's four-output runs, and
    planes of 10, 16 or 20 rows and at most 32 columns (the warp-per-plane kernel,
    its exact path taken by the plane holding NaN and -0)."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(h * 100 + w)
    x = torch.randn(n, c1, h, w, 16, generator=g).half()
    assert_bits_equal(ttn.sppf(x.to(device), 5), oops.sppf(x, 5))
    special = x.clone()
    bits = special.view(torch.int16)
    bits[0, 0, h // 2, w // 2, 3] = 0x7E05
    bits[-1, -1].masked_fill_(torch.rand(h, w, 16, generator=g) < 0.3, -0x8000)
    assert_bits_equal(ttn.sppf(special.to(device), 5), oops.sppf(special, 5))


@pytest.mark.parametrize("hw", [20, 7])
def test_sppf_nan_and_negative_zero_planes(device, hw):
    """Planes holding NaN (with payloads) or -0 take the exact per-lane CPU rule."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(19)
    x = torch.randn(2, 4, hw, hw, 16, generator=g).half()
    bits = x.view(torch.int16)
    bits[0, 1, hw // 2, 3 % hw, 5] = 0x7E05
    bits[0, 1, 0, 0, 6] = -0x0200  # 0xFE00
    bits[1, 2].masked_fill_(torch.rand(hw, hw, 16, generator=g) < 0.3, -0x8000)  # -0
    assert_bits_equal(ttn.sppf(x.to(device), 5), oops.sppf(x, 5))
