"""Shared pytest setup: the `gpu` marker, fp16 comparison helpers, golden data."""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libttn.so")


@pytest.fixture(scope="session")
def device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import thintnpu_b200
    thintnpu_b200.load()  # fails loudly if libttn.so is missing
    return torch.device("cuda", 0)


def half_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().reshape(-1).view(torch.int16).numpy().view(np.uint16)


def ordered(bits: np.ndarray) -> np.ndarray:
    """Map fp16 bit patterns to integers whose difference counts ulps (+0 == -0)."""
    b = bits.astype(np.int64)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> np.ndarray:
    """Per-element fp16 ulp distance; NaN positions must match (distance 0 there)."""
    ab, bb = half_bits(a), half_bits(b)
    nan_a = (ab & 0x7FFF) > 0x7C00
    nan_b = (bb & 0x7FFF) > 0x7C00
    assert np.array_equal(nan_a, nan_b), "NaN positions differ"
    d = np.abs(ordered(ab) - ordered(bb))
    d[nan_a] = 0
    return d


def ulp16(t: torch.Tensor) -> torch.Tensor:
    """Spacing of fp16 values at |t| (2^-24 in the subnormal range), as FP32."""
    a = t.float().abs()
    e = torch.floor(torch.log2(torch.clamp(a, min=2.0 ** -14)))
    return torch.pow(2.0, e - 10)


def check_bias_silu_residual(got, x, bias, residual, want):
    """Gate of the fused y = fp16(SiLU(x + b) + r) against CPU
    eager: |y - y_cpu| <= 2 fp16 ulp of y_cpu + 2^-18 |s| with s = SiLU(x + b) in
    FP32, and at least 99% of outputs bit-equal.  The second term is the FP32
    evaluation error of the SiLU value (CPU eager's own fp32 SiLU is not the
    correctly rounded formula: its exp is a low-accuracy polynomial), which the
    residual add passes on unscaled and which is many fp16 ulps of y wherever
    s + r nearly cancels.  Returns the bit-equal fraction."""
    got = got.detach().cpu()
    b = bias.float().view(1, x.size(1), 1, 1, 16)
    s = torch.nn.functional.silu(x.float() + b)
    err = (got.float() - want.float()).abs()
    bound = 2 * ulp16(want) + 2.0 ** -18 * s.abs()
    assert bool(torch.all(err <= bound)), float((err - bound).max())
    exact = float((got.view(torch.int16) == want.view(torch.int16)).float().mean())
    assert exact >= 0.99, exact
    return exact


def assert_bits_equal(a: torch.Tensor, b: torch.Tensor, what: str = "") -> None:
    assert a.shape == b.shape and a.dtype == b.dtype, (what, a.shape, b.shape, a.dtype, b.dtype)
    x = a.detach().cpu().contiguous().reshape(-1).view(torch.uint8)
    y = b.detach().cpu().contiguous().reshape(-1).view(torch.uint8)
    assert torch.equal(x, y), f"bit mismatch {what}"


def selection_index():
    return json.loads((GOLDEN / "selection_index.json").read_text())


def selection_case(name: str):
    with np.load(GOLDEN / "selection" / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}
