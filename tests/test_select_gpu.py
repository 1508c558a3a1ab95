"""GPU parity (bit-exact): YOLO26 detection selection.

* every reference fixture (verify_selection_flow.py:168-213, golden outputs of
  its CPU ``reference()``) in its layout, all 8 trace stages;
* BASELINE config 5 (logits with ties and NaNs, fused fp16 sigmoid, K =
  300/511/512/513, both modes, both NaN orders) against the numpy oracle run on
  CPU-eager sigmoid bits;
* eager == CUDA-graph replay, and replay after the input changed."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import selection_case, selection_index
from oracle import select as osel

pytestmark = pytest.mark.gpu


def to_half(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.float16)


def layout_view(x: torch.Tensor, layout: str, device) -> torch.Tensor:
    """Place x [B,A,C] on the device in the fixture's storage layout."""
    b, a, c = x.shape
    if layout == "contiguous":
        return x.contiguous().to(device)
    if layout == "transposed":
        return x.transpose(1, 2).contiguous().to(device).transpose(1, 2)
    if layout == "expanded":
        return x[:1].contiguous().to(device).expand(b, -1, -1)
    base = torch.zeros(b + 1, a * 2 + 2, c * 2 + 3, dtype=x.dtype)
    base[1:, 1:1 + 2 * a:2, 1:1 + 2 * c:2] = x
    return base.to(device)[1:, 1:1 + 2 * a:2, 1:1 + 2 * c:2]


def trace_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy().view(np.uint32)
    return t.numpy()


@pytest.mark.parametrize("case", [c["name"] for c in selection_index()])
def test_reference_fixture_bit_exact(device, case):
    import thintnpu_b200 as ttn
    meta = next(c for c in selection_index() if c["name"] == case)
    golden = selection_case(case)
    x = layout_view(to_half(golden["decoded"]), meta["layout"], device)
    trace = ttn.detection_select(x, meta["max_det"], meta["agnostic"], trace=True)
    oracle = osel.select(golden["decoded"], meta["max_det"], meta["agnostic"])
    for name, got in zip(osel.TRACE_NAMES, trace):
        have = trace_bits(got)
        want = oracle[name]
        assert have.shape == want.shape, (case, name, have.shape, want.shape)
        assert np.array_equal(have.astype(want.dtype), want), (case, name)
    eager = ttn.detection_select(x, meta["max_det"], meta["agnostic"])
    assert np.array_equal(trace_bits(eager), trace_bits(trace[0]))


def config5_logits(n: int, seed: int = 5, anchors: int = 8400, nc: int = 80) -> torch.Tensor:
    """Logits [n, 84, anchors] fp16 ~ N(-4, 2) (channel-planar, as decoded.transpose(1,2)
    sees them) with ~1% anchors copying another anchor's class row, some rows with
    equal values across classes, and a few NaNs (signs and payloads)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, 4 + nc, anchors, generator=g) * 2 - 4
    x[:, :4] = torch.rand(n, 4, anchors, generator=g) * 640
    x = x.half()
    for b in range(n):
        src = torch.randint(0, anchors, (anchors // 100,), generator=g)
        dst = torch.randint(0, anchors, (anchors // 100,), generator=g)
        x[b, 4:, dst] = x[b, 4:, src]
        rows = torch.randint(0, anchors, (anchors // 200,), generator=g)
        x[b, 4:, rows] = x[b, 4:5, rows]
        nans = torch.randint(0, anchors, (8,), generator=g)
        cls = torch.randint(0, nc, (8,), generator=g)
        payload = torch.tensor([0x7E00, 0xFE00, 0x7C01, 0xFD23] * 2, dtype=torch.int32).to(torch.int16)
        x.view(torch.int16)[b, 4 + cls, nans] = payload
    return x


@pytest.mark.parametrize("k", [300, 511, 512, 513])
@pytest.mark.parametrize("agnostic", [False, True])
@pytest.mark.parametrize("nan_last", [False, True])
def test_config5_fused_sigmoid_selection(device, k, agnostic, nan_last):
    import thintnpu_b200 as ttn
    logits = config5_logits(2)
    decoded_logits = logits.transpose(1, 2)  # [n, 8400, 84] view
    # oracle: CPU-eager fp16 sigmoid bits, then the stable selection order
    scores = decoded_logits.clone()
    scores[..., 4:] = torch.sigmoid(scores[..., 4:])
    bits = scores.contiguous().view(torch.int16).numpy().view(np.uint16)
    want = osel.select(bits, k, agnostic, nan_last)
    dev = logits.to(device).transpose(1, 2)
    got = ttn.detection_select(dev, k, agnostic, nan_last=nan_last, apply_sigmoid=True, trace=True)
    for name, t in zip(osel.TRACE_NAMES, got):
        have = trace_bits(t)
        assert np.array_equal(have.astype(want[name].dtype), want[name]), name
    # the unfused path: sigmoid kernel, then selection on scores
    sig = ttn.sigmoid(dev[..., 4:])
    dec = ttn.cat([dev[..., :4], sig], -1)
    plain = ttn.detection_select(dec, k, agnostic, nan_last=nan_last)
    assert np.array_equal(trace_bits(plain), want["output"])


def test_eager_equals_graph_replay_and_changed_input(device):
    import thintnpu_b200 as ttn
    logits = config5_logits(3, seed=9)
    scores = logits.clone()
    scores[:, 4:] = torch.sigmoid(scores[:, 4:])
    base = scores.to(device)
    x = base.transpose(1, 2)
    eager = ttn.detection_select(x, 300)
    ws = torch.empty(ttn.ops.workspace_size(3, 8400, 80, 300, 0), dtype=torch.uint8, device=device)
    ttn.detection_select(x, 300, workspace=ws)  # warm-up outside capture
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = ttn.detection_select(x, 300, workspace=ws)
    graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(trace_bits(eager), trace_bits(captured))
    changed = -scores
    base.copy_(changed.to(device))
    changed_eager = ttn.detection_select(x, 300)
    bits = changed.transpose(1, 2).contiguous().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(trace_bits(changed_eager), osel.select(bits, 300)["output"])
    graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(trace_bits(captured), trace_bits(changed_eager))


def test_batch_sharding_is_image_independent(device):
    """Images never interact: selecting a batch equals selecting each image."""
    import thintnpu_b200 as ttn
    logits = config5_logits(5, seed=21)
    dev = logits.to(device).transpose(1, 2)
    whole = trace_bits(ttn.detection_select(dev, 300, apply_sigmoid=True))
    for b in range(5):
        one = trace_bits(ttn.detection_select(dev[b:b + 1], 300, apply_sigmoid=True))
        assert np.array_equal(whole[b:b + 1], one)


def _pair_stage_logits(pattern: str) -> torch.Tensor:
    g = torch.Generator().manual_seed(31)
    if pattern == "config5":
        return config5_logits(2, seed=13)
    if pattern == "few_anchors":
        return config5_logits(2, seed=14, anchors=64)
    nc = 3 if pattern == "few_classes" else 80
    x = torch.randn(2, 4 + nc, 8400, generator=g) * 2 - 4
    x[:, :4] = torch.rand(2, 4, 8400, generator=g) * 640
    if pattern == "all_tied":
        x[:, 4:] = 0.5
    elif pattern == "many_high":  # fp16 sigmoid near 1 collapses many classes into ties
        x[:, 4:] = torch.randn(2, nc, 8400, generator=g) * 0.5 + 3
    x = x.half()
    if pattern == "nan_rows":
        flat = x.view(torch.int16)
        pick = torch.rand(2, nc, 8400, generator=g) < 0.05
        flat[:, 4:][pick] = torch.tensor(0x7E01, dtype=torch.int16)
        flat[:, 4:][pick & (torch.rand(2, nc, 8400, generator=g) < 0.5)] = torch.tensor(-0x0200, dtype=torch.int16)
    return x


@pytest.mark.parametrize("pattern", ["config5", "all_tied", "many_high", "nan_rows", "few_classes", "few_anchors"])
@pytest.mark.parametrize("nan_last", [False, True])
def test_class_aware_pair_stage_without_trace(device, pattern, nan_last):
    """Class-aware selection with the fused sigmoid and no trace (the one-kernel
    pair stage: candidate pairs from the second-best keys) against the oracle."""
    import thintnpu_b200 as ttn
    logits = _pair_stage_logits(pattern)
    view = logits.transpose(1, 2)
    scores = view.clone()
    scores[..., 4:] = torch.sigmoid(scores[..., 4:])
    bits = scores.contiguous().view(torch.int16).numpy().view(np.uint16)
    for k in (300, 7):
        want = osel.select(bits, k, False, nan_last)["output"]
        got = ttn.detection_select(logits.to(device).transpose(1, 2), k, nan_last=nan_last, apply_sigmoid=True)
        assert np.array_equal(trace_bits(got), want), (pattern, k)
