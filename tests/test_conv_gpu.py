"""GPU parity: the fused convolution (tcgen05 implicit GEMM, TMEM, TMA) against the
reference's conv + epilogue on the CPU: FP32 conv + bias, s / (1 + exp(-s)) in FP32,
one rounding to fp16 (convolution_native conv_flow.cpp:45-121).

The tensor cores sum the products in another order than the CPU conv, so an output
can round to a neighbouring fp16 value, and outputs near zero can differ by the FP32
accumulation error (proportional to sum |x| |w|).  Measured on the CPU: the reference
computation itself, with the input channels summed in a permuted order, moves by one
fp16 step plus at most 0.23 * 2^-23 * sum |x| |w| (20 seeded cases).  Gate: every
output within one fp16 step + 2^-21 * sum |x| |w|, and at least 99.5% - 5e-6 K of the
outputs bit-equal, K = ci * k * k products per output (measured on a B200: 99.98% at
K = 16, 99.7% at K = 576, 99.0% at K = 2304; the CPU with a permuted channel order
keeps 99.7% at K = 2304, so the tensor cores' FP32 accumulation is a little coarser
than sequential round-to-nearest adds)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import ops as oops

pytestmark = pytest.mark.gpu


def _case(b, ci, co, h, w, k, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, ci, h, w, generator=g).half()
    wt = (torch.randn(co, ci, k, k, generator=g) * (1.0 / (ci * k * k) ** 0.5)).half()
    bs = (torch.randn(co, generator=g) * 0.1).half() if bias else None
    return x, wt, bs


def _check(got_nchw, x, wt, bs, stride, silu):
    want = oops.conv2d(oops.pack_padded(x), wt, bs, stride, silu).float()
    got = got_nchw.cpu().float()
    k = wt.shape[-1]
    mag = F.conv2d(x.float().abs(), wt.float().abs(), None, stride=stride, padding=(k - 1) // 2)
    ulp = 2.0 ** torch.floor(torch.log2(want.abs().clamp(min=2.0 ** -14))) * 2.0 ** -10
    err = (got - want).abs()
    bound = ulp + mag * 2.0 ** -21
    assert torch.all(err <= bound), float((err - bound).max())
    exact = (got == want).float().mean().item()
    assert exact >= 0.995 - 5e-6 * wt.shape[1] * k * k, exact


def _run(device, b, ci, co, h, w, k, stride, silu=True, bias=True, nchw=False, seed=0):
    import thintnpu_b200 as ttn
    x, wt, bs = _case(b, ci, co, h, w, k, seed, bias)
    xd = oops.pack_padded(x).to(device)
    packed = ttn.conv2d_pack_weights(wt.to(device))
    assert torch.equal(packed.cpu(), oops.conv_pack_weights(wt))
    out = ttn.conv2d(xd, packed, None if bs is None else bs.to(device), co, k, stride, silu=silu, nchw=nchw)
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    got = out if nchw else oops.from_blocked(out.cpu())
    _check(got, x, wt, bs, stride, silu)


@pytest.mark.parametrize("b,ci,co,h,w,k,stride", [
    (2, 64, 128, 40, 40, 1, 1), (1, 32, 32, 80, 80, 1, 1), (3, 128, 256, 20, 20, 1, 1), (1, 128, 512, 20, 20, 1, 1),
    (2, 64, 64, 40, 40, 3, 1), (1, 16, 32, 20, 20, 3, 1), (2, 32, 64, 80, 80, 3, 2), (1, 256, 256, 20, 20, 3, 2),
    (1, 32, 48, 13, 13, 3, 1), (1, 32, 64, 13, 13, 3, 2), (1, 3, 32, 64, 64, 6, 2), (2, 80, 96, 24, 24, 3, 1),
    (1, 64, 64, 32, 32, 3, 1), (2, 32, 64, 80, 80, 3, 1)])  # halo tiles whose second sub-tile pads rows (80 -> 96)
def test_conv_matches_cpu(device, b, ci, co, h, w, k, stride):
    _run(device, b, ci, co, h, w, k, stride)


@pytest.mark.parametrize("b,ci,co,h,w", [(2, 3, 32, 64, 64), (1, 3, 16, 33, 47), (1, 16, 64, 40, 40), (1, 1, 48, 20, 21),
                                         (2, 5, 32, 17, 18), (1, 3, 32, 160, 160), (1, 2, 64, 31, 29),
                                         (3, 3, 48, 9, 9)])
def test_stem_conv_matches_cpu(device, b, ci, co, h, w):
    """One input channel block, 3x3 stride 2 (the YOLO stem): up to 3 real channels the
    tensor-core kernel (27-long reduction), more the CUDA-core kernel, which reads
    only the channels the weights use; odd sizes, 1 to 16 real channels, 16-64
    outputs."""
    _run(device, b, ci, co, h, w, 3, 2)
    _run(device, b, ci, co, h, w, 3, 2, silu=False, bias=False, seed=5)


def test_conv_without_bias_or_silu(device):
    _run(device, 2, 64, 64, 20, 20, 3, 1, silu=False, bias=False, seed=3)
    _run(device, 1, 32, 64, 40, 40, 1, 1, silu=False, bias=True, seed=4)


def test_conv_nchw_output(device):
    _run(device, 2, 64, 80, 20, 20, 1, 1, nchw=True, seed=5)  # the Detect terminals: co = 64 + 16 classes
    _run(device, 1, 32, 40, 20, 20, 3, 1, nchw=True, seed=6)


def test_conv_into_concat_slice(device):
    """out = a channel slice of a wider NC1HWC0 concat buffer (batch stride > one image)."""
    import thintnpu_b200 as ttn
    x, wt, bs = _case(2, 64, 64, 20, 20, 3, seed=7)
    buf = torch.full((2, 12, 20, 20, 16), 7.0, dtype=torch.float16, device=device)
    ttn.conv2d(oops.pack_padded(x).to(device), ttn.conv2d_pack_weights(wt.to(device)), bs.to(device), 64, 3, 1,
               out=buf[:, 4:8])
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    assert torch.all(buf[:, :4] == 7.0) and torch.all(buf[:, 8:] == 7.0)
    _check(oops.from_blocked(buf[:, 4:8].cpu()), x, wt, bs, 1, True)


def test_conv_rejects_unsupported(device):
    import thintnpu_b200 as ttn
    from thintnpu_b200._lib import TtnError
    x = torch.zeros(1, 2, 8, 8, 16, dtype=torch.float16, device=device)
    packed = torch.zeros(2, 25, 64, 16, dtype=torch.float16, device=device)
    with pytest.raises(TtnError, match="stride"):
        ttn.conv2d(x, packed, None, 64, 5, 1)
    with pytest.raises(TtnError, match="co % 16"):
        ttn.conv2d(x, torch.zeros(2, 1, 64, 16, dtype=torch.float16, device=device), None, 40, 1, 1)


# ---- residual epilogue and the C2f region (blocked_c2f.py:20-24) ----

@pytest.mark.parametrize("b,c,h,w", [(2, 128, 40, 40), (1, 32, 37, 23), (3, 64, 20, 20)])
def test_conv_residual_equals_conv_then_add(device, b, c, h, w):
    """The residual epilogue gives fp16(res + y) with y the plain conv's fp16 output:
    bit-identical to the conv followed by the separate fp16 add (the reference's
    y[-1] + value), also when the residual is the output buffer itself."""
    import thintnpu_b200 as ttn
    x, wt, bs = _case(b, c, c, h, w, 3, seed=c + h)
    g = torch.Generator().manual_seed(7)
    res = torch.randn(b, c // 16, h, w, 16, generator=g).half().to(device)
    xd, packed, bd = oops.pack_padded(x).to(device), ttn.conv2d_pack_weights(wt.to(device)), bs.to(device)
    plain = ttn.conv2d(xd, packed, bd, c, 3)
    want = ttn.add(res, plain)
    fused = ttn.conv2d(xd, packed, bd, c, 3, residual=res)
    inplace = res.clone()
    ttn.conv2d(xd, packed, bd, c, 3, out=inplace, residual=inplace)
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    assert torch.equal(fused.view(torch.int16), want.view(torch.int16))
    assert torch.equal(inplace.view(torch.int16), want.view(torch.int16))
    # and the add itself against the CPU rule, fp16(float(res) + float(y))
    cpu = (res.cpu().float() + plain.cpu().float()).half()
    assert torch.equal(fused.cpu().view(torch.int16), cpu.view(torch.int16))


def test_conv_residual_rejects_nchw(device):
    import thintnpu_b200 as ttn
    x = torch.zeros(1, 2, 8, 8, 16, dtype=torch.float16, device=device)
    packed = ttn.conv2d_pack_weights(torch.zeros(32, 32, 1, 1, dtype=torch.float16, device=device))
    with pytest.raises(Exception, match="NC1HWC0"):
        ttn.conv2d(x, packed, None, 32, 1, nchw=True, residual=torch.zeros(1, 32, 8, 8, dtype=torch.float16,
                                                                          device=device))


def _c2f_weights(c_in, c, n, c_out, seed):
    g = torch.Generator().manual_seed(seed)

    def conv(co, ci, k):
        return ((torch.randn(co, ci, k, k, generator=g) * (1.0 / (ci * k * k) ** 0.5)).half(),
                (torch.randn(co, generator=g) * 0.1).half())
    return conv(2 * c, c_in, 1), [(conv(c, c, 3), conv(c, c, 3)) for _ in range(n)], conv(c_out, (2 + n) * c, 1)


@pytest.mark.parametrize("b,c_in,c,n,c_out,hw", [(2, 256, 128, 2, 256, 40), (1, 64, 32, 1, 64, 80)])
def test_c2f_region_equals_reference_op_sequence(device, b, c_in, c, n, c_out, hw):
    """model.6's region (blocked_c2f.py:20-24; 256 -> 256 at 40x40, two bottlenecks) and
    a smaller one: the fused region against the same op sequence run op by op on the
    GPU (pack, conv, chunk, conv, conv, add, cat, conv, unpack), bit for bit, and
    against the CPU FP32 chain within fp16 accumulation noise."""
    import thintnpu_b200 as ttn
    from thintnpu_b200.yolo import C2fRegion
    cv1, m, cv2 = _c2f_weights(c_in, c, n, c_out, seed=c_in + n)
    dev = lambda wb: (wb[0].to(device), wb[1].to(device))
    region = C2fRegion(dev(cv1), [(dev(a), dev(bb)) for a, bb in m], dev(cv2))
    g = torch.Generator().manual_seed(11)
    x = torch.randn(b, c_in, hw, hw, generator=g).half()
    got = region(x.to(device))
    # op by op on the GPU, as blocked_forward does
    conv = lambda t, wb, k, nchw=False: ttn.conv2d(t, ttn.conv2d_pack_weights(wb[0].to(device)),
                                                    wb[1].to(device), wb[0].shape[0], k, nchw=nchw)
    y = list(conv(ttn.pack(x.to(device)), cv1, 1).chunk(2, 1))
    for a, bb in m:
        y.append(ttn.add(y[-1].contiguous(), conv(conv(y[-1].contiguous(), a, 3), bb, 3)))
    want = ttn.unpack(conv(torch.cat([t.contiguous() for t in y], 1), cv2, 1))
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # the CPU chain (FP32 convs, one fp16 rounding each, fp16 adds)
    ccv = lambda t, wb: oops.conv2d(oops.pack_padded(t), wb[0], wb[1], 1, True)
    ys = list(ccv(x, cv1).chunk(2, 1))
    for a, bb in m:
        ys.append((ys[-1].float() + ccv(ccv(ys[-1], a), bb).float()).half())
    cpu = ccv(torch.cat(ys, 1), cv2).float()
    diff = (got.cpu().float() - cpu).norm() / cpu.norm()
    assert diff < 2e-3, float(diff)


@pytest.mark.parametrize("ci,co,k,stride,bias", [(32, 64, 3, 2, True), (64, 80, 1, 1, False), (3, 32, 3, 2, True),
                                                  (128, 128, 3, 1, True)])
def test_aten_convolution_routing(device, ci, co, k, stride, bias):
    """aten::convolution (aten_adapter.cpp:106-112) routed to the tensor-core conv:
    F.conv2d / nn.Conv2d on fp16 CUDA tensors inside aten_routing(), NCHW in and out,
    no activation; the packed weight is reused while the weight is unchanged."""
    from thintnpu_b200 import aten
    x, wt, bs = _case(2, ci, co, 20, 24, k, 7 + ci, bias)
    conv = torch.nn.Conv2d(ci, co, k, stride, (k - 1) // 2, bias=bias).half().to(device).requires_grad_(False)
    with torch.no_grad():
        conv.weight.copy_(wt)
        if bias:
            conv.bias.copy_(bs)
    before = aten.ROUTED.get("aten::convolution", 0)
    with torch.inference_mode(), aten.aten_routing():
        got = conv(x.to(device))
        again = conv(x.to(device))
    assert aten.ROUTED["aten::convolution"] == before + 2
    assert torch.equal(got, again)
    _check(got, x, wt, bs, stride, silu=False)


def test_aten_convolution_rejects_unsupported(device):
    from thintnpu_b200 import aten
    x = torch.randn(1, 16, 8, 8, device=device).half()
    w = torch.randn(16, 16, 3, 3, device=device).half()
    with torch.inference_mode(), aten.aten_routing():
        with pytest.raises(RuntimeError, match="transposed/groups"):
            F.conv2d(x, w[:, :8], None, 1, 1, 1, 2)
        with pytest.raises(RuntimeError, match="dilation"):
            F.conv2d(x, w, None, 1, 2, 2)
        with pytest.raises(RuntimeError, match="k1/p0 stride 1 or k3/p1"):
            F.conv2d(x, torch.randn(16, 16, 5, 5, device=device).half(), None, 1, 2)
        y = F.conv2d(x.float(), w.float(), None, 1, 1)  # fp32 stays with PyTorch
    assert y.dtype == torch.float32


def test_torch_ops_conv_schemas(device):
    """thin_native_flow::conv / depthwise / pack_input and thin_blocked::conv
    (conv_flow.cpp:630-646, depthwise_flow.cpp:225-233, conv_blocked.cpp:198-210)."""
    import thintnpu_b200 as ttn
    from thintnpu_b200 import library  # noqa: F401
    nf, bl = torch.ops.thin_native_flow, torch.ops.thin_blocked
    x, wt, bs = _case(1, 64, 128, 16, 16, 3, 11)
    xb = nf.pack_input(x.to(device))
    assert torch.equal(xb.cpu(), oops.pack_padded(x))
    packed = ttn.conv2d_pack_weights(wt.to(device))
    y = nf.conv(xb, packed, bs.to(device), 128, 3, 1)
    _check(oops.from_blocked(y.cpu()), x, wt, bs, 1, True)
    y_nchw = nf.conv(xb, packed, bs.to(device), 128, 3, 2, False, True)
    _check(y_nchw, x, wt, bs, 2, False)
    y_blocked = bl.conv(xb, packed, bs.to(device), 128, 3, 1, False, True)
    assert torch.equal(y_blocked, y)
    with pytest.raises(RuntimeError, match="FP16 output"):
        bl.conv(xb, packed, bs.to(device), 128, 3, 1, True, True)
    xd = torch.randn(1, 4, 16, 16, 16, generator=torch.Generator().manual_seed(3)).half()
    wd = (torch.randn(64, 1, 3, 3, generator=torch.Generator().manual_seed(4)) / 3).half()
    got = nf.depthwise(xd.to(device), ttn.depthwise_pack_weights(wd.to(device)), None, 3, 1, False)
    assert torch.equal(got.cpu().view(torch.int16), oops.depthwise(xd, wd, None, 3, 1, False).view(torch.int16))


def test_bounded_wait_runs_out_and_is_reported(device):
    """Failure detection on the GPU without a fault: with the test hook armed, the
    next conv launch issues no input copy, so its MMA role (waiting for a ring stage)
    and its epilogue (waiting for an accumulator) wait on barriers that nothing
    signals.  Each gives up at its 200 ms limit, the fault word reports 1 | 4, the
    kernel frees its tensor memory with nothing in flight, the context stays usable,
    and the next call is correct."""
    import time

    import thintnpu_b200 as ttn
    from thintnpu_b200 import _lib
    x, wt, bs = _case(1, 32, 64, 8, 16, 3, 5)
    xd = oops.pack_padded(x).to(device)
    packed = ttn.conv2d_pack_weights(wt.to(device))
    b = bs.to(device)
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    _lib.lib().ttn_conv2d_test_withhold_copies()
    start = time.perf_counter()
    ttn.conv2d(xd, packed, b, 64, 3, 1)
    torch.cuda.synchronize()
    assert time.perf_counter() - start >= 0.15
    assert ttn.ops.conv2d_fault() == 5
    assert ttn.ops.conv2d_fault() == 0  # reading clears it
    out = ttn.conv2d(xd, packed, b, 64, 3, 1)
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    _check(oops.from_blocked(out.cpu()), x, wt, bs, 1, True)


def test_stem_conv_into_a_channel_slice(device):
    """The stem writing into channel blocks 1-2 of a wider buffer (batch stride past the
    dense image; 32-byte aligned rows) and into rows that are only 16-byte aligned:
    both bit-identical to the dense output, the blocks around them untouched."""
    import thintnpu_b200 as ttn
    x, wt, bs = _case(2, 3, 32, 48, 48, 3, 11)
    xd = oops.pack_padded(x).to(device)
    packed = ttn.conv2d_pack_weights(wt.to(device))
    dense = ttn.conv2d(xd, packed, bs.to(device), 32, 3, 2)
    wide = torch.full((2, 4, 24, 24, 16), 7.0, dtype=torch.float16, device=device)
    ttn.conv2d(xd, packed, bs.to(device), 32, 3, 2, out=wide[:, 1:3])
    flat = torch.full((2 * 4 * 24 * 24 * 16 + 8,), 7.0, dtype=torch.float16, device=device)
    shifted = flat[8:].view(2, 4, 24, 24, 16)  # 16 bytes past a 32-byte boundary
    ttn.conv2d(xd, packed, bs.to(device), 32, 3, 2, out=shifted[:, :2])
    torch.cuda.synchronize()
    assert ttn.ops.conv2d_fault() == 0
    assert torch.equal(wide[:, 1:3].view(torch.int16), dense.view(torch.int16))
    assert torch.equal(shifted[:, :2].view(torch.int16), dense.view(torch.int16))
    assert bool((wide[:, 0] == 7).all()) and bool((wide[:, 3] == 7).all())
    assert bool((shifted[:, 2:] == 7).all())
