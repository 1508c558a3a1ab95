"""GPU parity: depthwise conv against the reference's own FP32 operation order on the
CPU (depthwise_flow.cpp:60-162: acc = acc + x*w per tap in (ky, kx) order, + bias,
s/(1+exp(-s)), one rounding).  Without the SiLU the result is bit-exact; with it,
only the exp of the two math libraries differs: every output within one fp16 step
and at least 99.9% bit-equal."""
from __future__ import annotations

import pytest
import torch

from oracle import ops as oops

pytestmark = pytest.mark.gpu


def _case(b, c, h, w, k, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, c // 16, h, w, 16, generator=g).half()
    wt = (torch.randn(c, 1, k, k, generator=g) / k).half()
    bs = (torch.randn(c, generator=g) * 0.1).half() if bias else None
    return x, wt, bs


def _run(device, b, c, h, w, k, s, silu, bias=True, seed=0):
    import thintnpu_b200 as ttn
    x, wt, bs = _case(b, c, h, w, k, seed, bias)
    got = ttn.depthwise(x.to(device), ttn.depthwise_pack_weights(wt.to(device)),
                        None if bs is None else bs.to(device), k, s, silu=silu).cpu()
    want = oops.depthwise(x, wt, bs, k, s, silu)
    return got, want


@pytest.mark.parametrize("b,c,h,w,k,s", [(2, 64, 40, 40, 3, 1), (1, 128, 20, 20, 3, 2), (1, 32, 80, 80, 5, 1),
                                         (3, 16, 13, 13, 7, 2), (1, 256, 20, 20, 1, 1), (2, 48, 160, 160, 3, 1)])
def test_depthwise_unfused_bit_exact(device, b, c, h, w, k, s):
    got, want = _run(device, b, c, h, w, k, s, silu=False, seed=k + s)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("b,c,h,w,k,s", [(2, 64, 40, 40, 3, 1), (1, 128, 20, 20, 3, 2), (2, 48, 160, 160, 3, 1)])
def test_depthwise_silu_matches_cpu(device, b, c, h, w, k, s):
    got, want = _run(device, b, c, h, w, k, s, silu=True, seed=3)
    g, wv = got.float(), want.float()
    ulp = 2.0 ** torch.floor(torch.log2(wv.abs().clamp(min=2.0 ** -14))) * 2.0 ** -10
    assert torch.all((g - wv).abs() <= ulp)
    assert (g == wv).float().mean().item() >= 0.999


def test_depthwise_without_bias(device):
    got, want = _run(device, 1, 32, 24, 24, 3, 1, silu=False, bias=False, seed=9)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_depthwise_silu_every_fp16_input(device):
    """1x1 kernel, weight 1, no bias: the accumulator is each fp16 value itself, so the
    SiLU epilogue sees all 65,536 inputs (NaNs, infinities, subnormals, signed zeros)."""
    import thintnpu_b200 as ttn
    x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.float16).reshape(1, 16, 16, 16, 16)
    wt = torch.ones(256, 1, 1, 1, dtype=torch.float16)
    got = ttn.depthwise(x.to(device), ttn.depthwise_pack_weights(wt.to(device)), None, 1, 1, silu=True).cpu()
    want = oops.depthwise(x, wt, None, 1, 1, True)
    g, wv = got.float(), want.float()
    nan = torch.isnan(wv)
    assert torch.equal(torch.isnan(g), nan)
    g, wv = g[~nan], wv[~nan]
    assert torch.equal(torch.isinf(g), torch.isinf(wv))
    fin = torch.isfinite(wv)
    ulp = 2.0 ** torch.floor(torch.log2(wv[fin].abs().clamp(min=2.0 ** -14))) * 2.0 ** -10
    assert torch.all((g[fin] - wv[fin]).abs() <= ulp)
    assert (g == wv).float().mean().item() >= 0.999


@pytest.mark.parametrize("scale", [0.01, 1.0, 6.0, 30.0])
def test_depthwise_silu_rounds_like_fp32_silu(device, scale):
    """The epilogue's fast SiLU either settles a value by its error bracket or takes
    the IEEE-divide path, so every output must equal fp16(silu(acc)) computed by the
    library's FP32 SiLU.  With a 1x1 kernel and no bias, acc = x * w exactly (two fp16
    values), which gives FP32 accumulators of every magnitude at the chosen scale."""
    import thintnpu_b200 as ttn
    g = torch.Generator().manual_seed(int(scale * 100))
    x = (torch.randn(2, 8, 32, 32, 16, generator=g) * scale).half()
    wt = torch.randn(128, 1, 1, 1, generator=g).half()
    xd, wd = x.to(device), wt.to(device)
    got = ttn.depthwise(xd, ttn.depthwise_pack_weights(wd), None, 1, 1, silu=True)
    acc = xd.float() * wd.float().reshape(1, 8, 1, 1, 16) + 0.0  # 0 + x*w: a -0 product sums to +0
    want = ttn.silu(acc).half()
    bad = got.view(torch.int16) != want.view(torch.int16)
    assert not bad.any(), (int(bad.sum()), acc[bad][:4].tolist(), got[bad][:4].tolist(), want[bad][:4].tolist())
