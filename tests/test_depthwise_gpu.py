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
