"""GPU parity: the fused C2PSA attention (tcgen05 tensor cores, TMEM) against the
reference's chain in CPU eager fp16 -- q^T @ k, * scale, softmax, v @ attn^T
(whole_blocked.py:91-110), every op rounding to fp16.

The GPU accumulates both products in FP32 in a different order from the CPU
GEMM, so an fp16 rounding of a score or an output can land one step away.  A
score that lands one fp16 step away changes its softmax weight by that step
(relative), which moves an output by up to the step of the row's largest |z|
times the channel's largest |v|: the reference chain run with another FP32
summation order moves by up to 0.25 of that over 30 seeded trials (std 0.5 to
4).  Gate: every output within 1e-3 + |want| 2^-8 + max|v| * ulp16(max|z|) of
the CPU value, and at least 97% bit-equal."""
from __future__ import annotations

import pytest
import torch

from oracle import ops as oops

pytestmark = pytest.mark.gpu


def _qkv(b, heads, kd, hd, n, seed, std=1.0):
    """The qkv conv output [B, heads*(2kd+hd), N] and its q, k, v split views."""
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(b, heads * (2 * kd + hd), n, generator=g) * std).half()
    q, k, v = qkv.view(b, heads, 2 * kd + hd, n).split([kd, kd, hd], dim=2)
    return qkv, q, k, v


def _check(got, want, q, k, v, scale):
    got = got.cpu().float()
    want = want.float()
    err = (got - want).abs()
    zmax = ((q.float().transpose(-2, -1) @ k.float()) * scale).abs().amax(-1)  # [B, heads, N] per query
    ulp = torch.exp2(torch.floor(torch.log2(zmax.clamp(min=2.0 ** -14)))) * 2.0 ** -10
    vmax = v.float().abs().amax(-1)  # [B, heads, hd] per channel
    bound = 1e-3 + want.abs() * 2.0 ** -8 + vmax[..., :, None] * ulp[..., None, :]
    assert torch.all(err <= bound), float((err - bound).max())
    exact = (got == want).float().mean().item()
    assert exact >= 0.97, exact


@pytest.mark.parametrize("b,heads,kd,hd,n", [(2, 4, 32, 64, 400), (1, 2, 16, 32, 64), (1, 1, 64, 128, 256),
                                             (2, 2, 32, 64, 200), (1, 1, 32, 64, 448), (1, 2, 64, 64, 448),
                                             (3, 1, 16, 96, 40), (48, 4, 32, 64, 400)])
def test_attention_matches_cpu_chain(device, b, heads, kd, hd, n):
    import thintnpu_b200 as ttn
    scale = kd ** -0.5
    qkv, q, k, v = _qkv(b, heads, kd, hd, n, seed=n + kd)
    dev = qkv.to(device)
    dq, dk, dv = dev.view(b, heads, 2 * kd + hd, n).split([kd, kd, hd], dim=2)
    got = ttn.attention(dq, dk, dv, scale)
    torch.cuda.synchronize()
    assert ttn.ops.attention_fault() == 0
    _check(got, oops.attention(q, k, v, scale), q, k, v, scale)


@pytest.mark.parametrize("b,heads,kd,hd,n", [(2, 4, 32, 64, 400), (1, 2, 64, 64, 448), (48, 4, 32, 64, 400)])
def test_attention_prescale_matches_cpu_chain(device, b, heads, kd, hd, n):
    """The YOLO26 order (attention_scale_before_matmul, whole_blocked.py:96-99):
    the query is rounded to fp16(q * scale) before the product."""
    import thintnpu_b200 as ttn
    scale = kd ** -0.5
    qkv, q, k, v = _qkv(b, heads, kd, hd, n, seed=7 * n + kd)
    dev = qkv.to(device)
    dq, dk, dv = dev.view(b, heads, 2 * kd + hd, n).split([kd, kd, hd], dim=2)
    got = ttn.attention(dq, dk, dv, scale, prescale=True)
    torch.cuda.synchronize()
    assert ttn.ops.attention_fault() == 0
    want = oops.attention(q, k, v, scale, prescale=True)
    assert not torch.equal(want, oops.attention(q, k, v, scale))  # the two orders differ on these inputs
    _check(got, want, q, k, v, scale)
    assert torch.equal(dev, qkv.to(device))  # the input is not modified (q is scaled in shared memory)


def test_attention_contiguous_inputs_and_out_view(device):
    import thintnpu_b200 as ttn
    _, q, k, v = _qkv(2, 4, 32, 64, 400, seed=3, std=2.0)
    out = torch.zeros(2, 4, 64, 408, dtype=torch.float16, device=device)[..., :400]
    ttn.attention(q.contiguous().to(device), k.contiguous().to(device), v.contiguous().to(device), 32 ** -0.5,
                  out=out)
    torch.cuda.synchronize()
    assert ttn.ops.attention_fault() == 0
    _check(out, oops.attention(q, k, v, 32 ** -0.5), q, k, v, 32 ** -0.5)


def test_attention_nan_and_inf_rows(device):
    """A NaN or +inf in a query's scores makes the reference's softmax row NaN
    (exp(x - max) is NaN there); the output row is NaN in both."""
    import thintnpu_b200 as ttn
    qkv, q, k, v = _qkv(1, 2, 32, 64, 96, seed=5)
    q[0, 0, 3, 7] = float("nan")
    q[0, 1, :, 11] = 60000.0  # scores overflow fp16 to +-inf
    want = oops.attention(q, k, v, 32 ** -0.5)
    dev = qkv.to(device)
    dq, dk, dv = dev.view(1, 2, 128, 96).split([32, 32, 64], dim=2)
    got = ttn.attention(dq, dk, dv, 32 ** -0.5).cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    finite = ~torch.isnan(want)
    assert torch.isnan(want).any()
    assert torch.allclose(got[finite].float(), want[finite].float(), atol=2e-3, rtol=2 ** -7)


def test_attention_rejects_unsupported_shapes(device):
    import thintnpu_b200 as ttn
    from thintnpu_b200._lib import TtnError
    q = torch.zeros(1, 1, 32, 500, dtype=torch.float16, device=device)
    v = torch.zeros(1, 1, 64, 500, dtype=torch.float16, device=device)
    with pytest.raises(TtnError, match="tokens"):
        ttn.attention(q, q, v, 1.0)  # 500 tokens + 64 > 512 TMEM columns
    q = torch.zeros(1, 1, 24, 64, dtype=torch.float16, device=device)
    with pytest.raises(TtnError, match="key_dim"):
        ttn.attention(q, q, v[..., :64], 1.0)
