"""GPU parity: SiLU, sigmoid, add/sub/mul/div, and the fused config-1 op vs CPU eager.

Tolerances (north star): fp16 elementwise within 2 ulp of PyTorch CPU eager;
SiLU and sigmoid are held to bit equality (the kernels reproduce CPU's FP32
formula and its rounding), binary ops with alpha == 1 as well.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import assert_bits_equal, check_bias_silu_residual, half_bits, ulp_diff
from oracle import ops as oops

pytestmark = pytest.mark.gpu

ALL_HALVES = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.float16)


@pytest.mark.parametrize("name", ["silu", "sigmoid"])
def test_unary_exhaustive_fp16_bit_exact(device, name):
    import thintnpu_b200 as ttn
    fn = getattr(ttn, name)
    ref = getattr(oops, name)(ALL_HALVES)
    # dense aligned arithmetic path, an odd-length tail, and a strided view
    assert_bits_equal(fn(ALL_HALVES.to(device)), ref, name)
    odd = ALL_HALVES[3:].clone()
    assert_bits_equal(fn(odd.to(device)), getattr(oops, name)(odd), name + " tail")
    strided = ALL_HALVES.view(256, 256).t()
    assert_bits_equal(fn(strided.to(device)), getattr(oops, name)(strided), name + " strided")
    # dense table path (>= 2^25 elements), with a tail, in place and out of place
    big = ALL_HALVES.repeat(520)[5:]
    want = ref.repeat(520)[5:]
    assert_bits_equal(fn(big.to(device)), want, name + " table")
    if name == "silu":
        inplace = big.to(device)
        ttn.silu_(inplace)
        assert_bits_equal(inplace, want, name + " table in place")


@pytest.mark.parametrize("path", ["table", "arithmetic"])
@pytest.mark.parametrize("name", ["silu", "sigmoid"])
def test_unary_all_input_pairs_bit_exact(device, name, path):
    """Every ordered pair of fp16 inputs in one 32-bit word, 2^32 pairs in 16
    launches of 2^28.  The arithmetic core computes the two lanes of a word
    together (one shared reciprocal), so its result is a function of the pair;
    views with three outer dims take that kernel, dense tensors the table kernel."""
    import thintnpu_b200 as ttn
    fn = getattr(ttn, name)
    table = getattr(oops, name)(ALL_HALVES).view(torch.int16).to(device)  # CPU result per input bits
    rows = 4096
    if path == "table":  # dense
        x = torch.empty(rows, 65536, 2, dtype=torch.int16, device=device)
    else:  # gaps at three levels: the general row kernel (three outer dims)
        buf = torch.empty(rows // 4, 3, 3, 65536 + 8, 2, dtype=torch.int16, device=device)
        x = buf[:, :2, :2, :65536]
    x[..., 0] = torch.arange(65536, dtype=torch.int32, device=device).to(torch.int16)
    for h0 in range(0, 65536, rows):
        hi = torch.arange(h0, h0 + rows, dtype=torch.int32, device=device).to(torch.int16)
        x[..., 1] = hi.view(x.shape[:-2])[..., None]
        y = fn(x.view(torch.float16)).view(torch.int16).reshape(rows, 65536, 2)
        bad = (y[..., 0] != table[None, :]) | (y[..., 1] != table[h0:h0 + rows, None])
        if bool(bad.any()):
            r, c = (int(v) for v in bad.nonzero()[0])
            raise AssertionError(f"{name}/{path}: pair (lo=0x{c:04x}, hi=0x{h0 + r:04x}) -> "
                                 f"{int(y[r, c, 0]) & 0xffff:04x},{int(y[r, c, 1]) & 0xffff:04x}, "
                                 f"want {int(table[c]) & 0xffff:04x},{int(table[h0 + r]) & 0xffff:04x}")


@pytest.mark.parametrize("rows", ["one outer dim", "two outer dims"])
def test_unary_row_family_table_path(device, rows):
    """Channel slices of a batch (the zero-copy concat views): 16-byte rows with
    one or two outer dims and >= 2^22 vectors take the row-family table kernel."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(17)
    base = (torch.randn(16, 96, 160, 160, generator=g) * 4).half()
    def view(t):
        return t[:, 4:92] if rows == "one outer dim" else t.view(16, 96, 25600)[:, 4:92, :25592]
    dev = base.to(device)
    ttn.silu_(view(dev))
    want = base.clone()
    want_view = view(want)
    want_view.copy_(oops.silu(want_view.contiguous()))
    assert_bits_equal(dev, want, rows)
    got = ttn.sigmoid(view(base.to(device)))
    assert_bits_equal(got, oops.sigmoid(view(base).contiguous()), rows + " sigmoid")


@pytest.mark.parametrize("shape", [(1,), (3,), (7,), (100,), (2047,), (2048,), (2049,), (16385,),
                                   (65537,), (0,), (), (3, 5, 7)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_binary_sizes(device, shape, dtype):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(42)
    a = (torch.rand(shape, generator=g) * 2 - 1).to(dtype)
    b = (torch.rand(shape, generator=g) + 0.5).to(dtype)
    for op in ("add", "sub", "mul", "div"):
        got = getattr(ttn, op)(a.to(device), b.to(device)).cpu()
        want = oops.binary(op, a, b)
        if dtype == torch.float16:
            assert_bits_equal(got, want, f"{op} {shape}")
        else:
            torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)


def test_binary_alpha_strided_broadcast(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(7)
    a = torch.randn(2, 5, 7, generator=g).half()
    b = torch.randn(2, 5, 7, generator=g).half() + 2
    for op in ("sub", "mul", "div"):
        got = getattr(ttn, op)(a.to(device).transpose(0, 2), b.to(device).transpose(0, 2))
        assert_bits_equal(got, oops.binary(op, a.transpose(0, 2), b.transpose(0, 2)), op)
    for alpha in (2.0, -0.5):
        got = ttn.sub(a.to(device), b.to(device), alpha=alpha)
        assert ulp_diff(got, torch.sub(a, b, alpha=alpha)).max() <= 2
    # row, column and scalar broadcast; narrow [...,2] box slices (verify_narrow_binary.py)
    x = torch.randn(1, 3, 9, 11, 16, generator=g).half()
    row = torch.randn(1, 1, 1, 11, 16, generator=g).half()
    col = torch.randn(1, 3, 9, 1, 1, generator=g).half()
    for other in (row, col, torch.tensor(1.5, dtype=torch.float16)):
        got = ttn.add(x.to(device), other.to(device))
        assert_bits_equal(got, x + other, "broadcast")
    got = ttn.mul(x.to(device)[..., 2:4], x.to(device)[..., :2])
    assert_bits_equal(got, x[..., 2:4] * x[..., :2], "narrow")
    got = ttn.mul(x.to(device), 32 ** -0.5)
    assert_bits_equal(got, x * 32 ** -0.5, "python scalar")


def test_silu_inplace_on_strided_parent_and_c2f_chain(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(42)
    a = torch.randn(2, 7, 5, 7, generator=g).half()
    x = a.to(device)
    part = torch.split(x, [3, 4], 1)[1]
    ptr = part.data_ptr()
    out = ttn.silu_(part)
    assert out is part and out.data_ptr() == ptr
    ref = a.clone()
    F.silu(torch.split(ref, [3, 4], 1)[1], inplace=True)
    assert_bits_equal(x, ref, "silu_ strided parent")
    for channels in (8, 7):
        a = torch.randn(2, channels, 13, 11, generator=g).half() * 0.5
        x = a.to(device)
        p, q = torch.split(x, [channels // 2, channels - channels // 2], 1)
        rp, rq = torch.split(a.clone(), [channels // 2, channels - channels // 2], 1)
        ttn.silu_(q)
        F.silu(rq, inplace=True)
        z = ttn.cat((p, ttn.add(q, q)), 1)
        assert_bits_equal(z, torch.cat((rp, rq + rq), 1), "c2f chain")


def test_add_silu_every_input_bit_exact(device):
    """a + SiLU(raw): raw over all 65,536 fp16 patterns (twice, against two random a),
    bit-identical to CPU eager SiLU then the fp16 add wherever that sum is a number,
    and to ttn's own silu then add where it is NaN (NaN or -inf raw: the device add
    returns its canonical NaN, as ttn_binary does); dense, then NC1HWC0 channel slices
    of wider buffers (batch-strided rows), then a layout that takes the silu-then-add
    fallback (rows of 12 elements)."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(3)
    raw = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.float16).repeat(2)
    a = (torch.randn(raw.numel(), generator=g) * 4).half()
    want = a + oops.silu(raw)
    got = ttn.ops.add_silu(a.to(device), raw.to(device)).cpu()
    number = ~torch.isnan(want)
    assert_bits_equal(got[number], want[number], "dense")
    two_step = ttn.add(a.to(device), ttn.silu(raw.to(device))).cpu()
    assert torch.isnan(got[~number]).all()
    assert_bits_equal(got[~number], two_step[~number], "dense NaN")
    wide_a = (torch.randn(3, 6, 20, 20, 16, generator=g) * 2).half()
    wide_raw = (torch.randn(3, 4, 20, 20, 16, generator=g) * 3).half()
    out = torch.zeros(3, 8, 20, 20, 16, dtype=torch.float16, device=device)
    da, draw = wide_a.to(device), wide_raw.to(device)
    ttn.ops.add_silu(da[:, 1:3], draw[:, 2:4], out=out[:, 4:6])
    assert_bits_equal(out[:, 4:6], wide_a[:, 1:3] + oops.silu(wide_raw[:, 2:4]), "channel slices")
    assert torch.count_nonzero(out[:, :4]) == 0 and torch.count_nonzero(out[:, 6:]) == 0
    odd_a = (torch.randn(5, 12, generator=g)).half()
    odd_raw = (torch.randn(5, 16, generator=g) * 3).half()[:, :12]
    got = ttn.ops.add_silu(odd_a.to(device), odd_raw.to(device))
    assert_bits_equal(got, odd_a + oops.silu(odd_raw), "fallback layout")


def test_config1_bias_silu_residual(device):
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(1)
    x = oops.to_blocked(torch.randn(1, 128, 80, 80, generator=g).half())
    r = oops.to_blocked(torch.randn(1, 128, 80, 80, generator=g).half())
    b = (torch.randn(128, generator=g) * 0.1).half()
    got = ttn.bias_silu_residual(x.to(device), b.to(device), r.to(device))
    check_bias_silu_residual(got, x, b, r, oops.bias_silu_residual(x, b, r))


@pytest.mark.parametrize("dtype", [torch.float32])
def test_unary_float32(device, dtype):
    import thintnpu_b200 as ttn
    a = torch.linspace(-8, 8, 65537, dtype=dtype)
    torch.testing.assert_close(ttn.sigmoid(a.to(device)).cpu(), torch.sigmoid(a), rtol=2e-6, atol=1e-7)
    torch.testing.assert_close(ttn.silu(a.to(device)).cpu(), F.silu(a), rtol=2e-6, atol=1e-7)


def test_unary_nan_payloads_follow_cpu(device):
    import thintnpu_b200 as ttn
    vals = [0x7E00, 0xFE00, 0x7C01, 0x7D23, 0xFD23, 0x7FFF, 0xFFFF, 0x7C00, 0xFC00]
    h = torch.tensor(vals, dtype=torch.int32).to(torch.int16).view(torch.float16)
    assert np.array_equal(half_bits(ttn.sigmoid(h.to(device))), half_bits(torch.sigmoid(h)))
    assert np.array_equal(half_bits(ttn.silu(h.to(device))), half_bits(F.silu(h)))
