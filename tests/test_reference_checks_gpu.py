"""GPU: the checks of the reference's acceptance scripts, run through the drop-in.

Each test restates the cases and tolerances of one reference script --
verify_ops.py (binary ops, cat/split, in-place SiLU and its C2f chain, views),
verify_flow_ops.py (blocked max-pool and upsample), verify_cat.py (bitwise
concat), verify_softmax.py (softmax shapes, shifts, views, non-finite rows,
half_to_float) and verify_graph.py (CapturedForward semantics) -- against
``import thin_backend`` with the reference's ``npu`` device mapped to
``thin_backend.device`` (cuda) and ATen routing on, and checks that every op
class the script exercises was routed to libttn (``aten.ROUTED``)."""
from __future__ import annotations

import gc
import math
import threading

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture
def tb(device):
    import thin_backend
    with torch.inference_mode(), thin_backend.aten_routing():
        yield thin_backend


def _compare(actual, expected, atol=0.0):
    assert actual.device.type == "cuda"
    got = actual.cpu()
    assert got.shape == expected.shape and got.dtype == expected.dtype
    assert bool(torch.isfinite(got).all())
    err = (got.float() - expected.float()).abs().max().item() if got.numel() else 0.0
    assert err <= atol, (tuple(got.shape), got.dtype, err, atol)


def _alias(view, base):
    assert view.untyped_storage().data_ptr() == base.untyped_storage().data_ptr()


def test_verify_ops_checks(tb):
    dev = tb.device
    g = torch.Generator().manual_seed(42)
    for dtype, tol in ((torch.float32, 1e-5), (torch.float16, 1e-3)):
        for shape in ((1,), (3,), (7,), (100,), (2047,), (2048,), (2049,), (16385,), (65537,), (0,), (), (3, 5, 7)):
            a = torch.rand(shape, generator=g).to(dtype) * 2 - 1
            b = torch.rand(shape, generator=g).to(dtype) + 0.5
            for op in ("sub", "mul", "div"):
                _compare(getattr(torch, op)(a.to(dev), b.to(dev)), getattr(torch, op)(a, b), tol)
        a = torch.rand(2, 5, 7, generator=g).to(dtype)
        b = torch.rand(2, 5, 7, generator=g).to(dtype) + 0.5
        for op in ("sub", "mul", "div"):
            _compare(getattr(torch, op)(a.to(dev).transpose(0, 2), b.to(dev).transpose(0, 2)),
                     getattr(torch, op)(a.transpose(0, 2), b.transpose(0, 2)), tol)
        _compare(torch.sub(a.to(dev), b.to(dev), alpha=2), torch.sub(a, b, alpha=2), tol)
    for dtype in (torch.float32, torch.float16):  # cat / split
        for dim in (0, 1, 2, -1):
            shape_b = [3, 5, 7]
            shape_b[dim % 3] = 4
            a, b = torch.randn(3, 5, 7, generator=g).to(dtype), torch.randn(shape_b, generator=g).to(dtype)
            _compare(torch.cat((a.to(dev), b.to(dev), a.to(dev)), dim), torch.cat((a, b, a), dim))
        a = torch.randn(2, 5, 7, generator=g).to(dtype)
        x = a.to(dev)
        for dim in (0, 1, 2, -1):
            parts, refs = torch.split(x, 2, dim), torch.split(a, 2, dim)
            assert len(parts) == len(refs)
            for p, r in zip(parts, refs):
                _alias(p, x)
                _compare(p, r)
            _compare(torch.cat(parts, dim), a)
            sizes = [1, 0, a.shape[dim] - 1]
            for p, r in zip(torch.split(x, sizes, dim), torch.split(a, sizes, dim)):
                _alias(p, x)
                _compare(p, r)
        xt = a.to(dev).transpose(0, 2)
        _compare(torch.cat((xt, xt), 1), torch.cat((a.transpose(0, 2), a.transpose(0, 2)), 1))
        empty = torch.empty(0, dtype=dtype)
        _compare(torch.cat((empty.to(dev), a.to(dev), empty.to(dev)), 1), a)
        _compare(torch.cat((empty.to(dev), empty.to(dev))), torch.empty(0, dtype=dtype))
    for dtype, tol in ((torch.float32, 1e-5), (torch.float16, 1e-3)):  # in-place SiLU and the C2f chain
        for shape in ((1,), (3,), (7,), (100,), (2049,), (65537,), (0,), (), (2, 7, 5, 7)):
            count = math.prod(shape)
            a = torch.linspace(-4, 4, max(1, count)).to(dtype)[:count].reshape(shape)
            x = a.to(dev)
            pointer = x.data_ptr()
            out = F.silu(x, inplace=True)
            assert out is x and x.data_ptr() == pointer
            _compare(out, F.silu(a), tol)
        a = torch.randn(2, 7, 5, 7, generator=g).to(dtype)
        x = a.to(dev)
        part, ref_part = torch.split(x, [3, 4], 1)[1], torch.split(a, [3, 4], 1)[1]
        pointer = part.data_ptr()
        out = F.silu(part, inplace=True)
        F.silu(ref_part, inplace=True)
        assert out is part and out.data_ptr() == pointer
        _compare(x, a, tol)
        for channels in (8, 7):
            a = torch.randn(2, channels, 13, 11, generator=g).to(dtype) * 0.5
            x = a.to(dev)
            half = [channels // 2, channels - channels // 2]
            p, q = torch.split(x, half, 1)
            rp, rq = torch.split(a, half, 1)
            F.silu(q, inplace=True)
            F.silu(rq, inplace=True)
            _compare(torch.cat((p, torch.add(q, q)), 1), torch.cat((rp, torch.add(rq, rq)), 1), tol)
            _compare(x, a, tol)
    for dtype in (torch.float32, torch.float16):  # views alias and keep strides
        a = torch.randn(2, 3, 7, generator=g).to(dtype)
        x = a.to(dev)
        for y, r in ((x.view(6, 7), a.view(6, 7)), (x.transpose(0, 2), a.transpose(0, 2)),
                     (x.unsqueeze(1), a.unsqueeze(1)),
                     (x.unsqueeze(0).expand(4, -1, -1, -1), a.unsqueeze(0).expand(4, -1, -1, -1)),
                     (x.as_strided((2, 3), (21, 7), 1), a.as_strided((2, 3), (21, 7), 1))):
            _alias(y, x)
            assert y.stride() == r.stride() and y.storage_offset() == r.storage_offset()
            _compare(y, r)
        y = x.unsqueeze(0).expand(2, -1, -1, -1)
        _compare(torch.cat((y, y), -1), torch.cat((a.unsqueeze(0).expand(2, -1, -1, -1),) * 2, -1))


def test_verify_ops_checks_were_routed(device):
    import thin_backend
    from thintnpu_b200 import aten
    before = dict(aten.ROUTED)
    with torch.inference_mode(), thin_backend.aten_routing():
        x = torch.rand(7, device=thin_backend.device).half()
        torch.sub(x, x)
        torch.mul(x, x)
        torch.div(x, x + 1)
        torch.cat((x, x))
        F.silu(x, inplace=True)
    for name in ("aten::sub", "aten::mul", "aten::div", "aten::add", "aten::cat", "aten::silu_"):
        assert aten.ROUTED.get(name, 0) > before.get(name, 0), name


def _to_blocked(x):
    n, c, h, w = x.shape
    return x.reshape(n, c // 16, 16, h, w).permute(0, 1, 3, 4, 2).contiguous()


def _from_blocked(y):
    n, c1, h, w, _ = y.shape
    return y.permute(0, 1, 4, 2, 3).reshape(n, c1 * 16, h, w).contiguous()


def test_verify_flow_ops_checks(tb):
    """Blocked max-pool and upsample, bit-exact against CPU F.max_pool2d (FP32) and
    F.interpolate nearest (verify_flow_ops.py)."""
    dev = tb.device
    g = torch.Generator().manual_seed(0)
    for c, h, w, k in ((256, 20, 20, 5), (128, 40, 40, 5), (512, 20, 20, 5), (32, 13, 17, 3), (16, 7, 9, 7),
                       (48, 1, 31, 5)):
        x = torch.randn(1, c, h, w, generator=g).half()
        got = _from_blocked(torch.ops.thin_native_flow.maxpool(_to_blocked(x).to(dev), k).cpu())
        want = F.max_pool2d(x.float(), k, stride=1, padding=k // 2).half()
        assert torch.equal(got, want), (c, h, w, k)
    for c, h, w in ((128, 40, 40), (256, 20, 20), (64, 13, 17), (16, 1, 33)):
        x = torch.randn(1, c, h, w, generator=g).half()
        got = _from_blocked(torch.ops.thin_native_flow.upsample(_to_blocked(x).to(dev)).cpu())
        assert torch.equal(got, F.interpolate(x.float(), scale_factor=2, mode="nearest").half()), (c, h, w)


def test_verify_cat_checks(tb):
    """Bitwise concat over dims, sizes, offsets, transposes, splits, expands,
    empties and special values (verify_cat.py)."""
    dev = tb.device
    g = torch.Generator().manual_seed(42)
    cases = [0]

    def check(cpu, parts, dim):
        actual = torch.cat(parts, dim)
        assert actual.device.type == "cuda" and actual.is_contiguous()
        expected = torch.cat(cpu, dim)
        bits = torch.int16 if actual.dtype == torch.float16 else torch.int32
        assert torch.equal(actual.cpu().view(bits), expected.view(bits)), (dim, [list(t.shape) for t in cpu])
        cases[0] += 1

    for dtype in (torch.float16, torch.float32):
        for dim in range(4):
            for outer in (1, 3):
                inputs = []
                for size in (1, 2, 5):
                    shape = [outer, 3, 32, 32]
                    shape[dim] = size if dim != 3 else size * 32
                    inputs.append(torch.randn(shape, generator=g).to(dtype))
                check(inputs, [t.to(dev) for t in inputs], dim)
        for length in (16, 8192, 16384, 16384 + 16, 131072 + 16):
            inputs = [torch.randn(3, length, generator=g).to(dtype) for _ in range(3)]
            check(inputs, [t.to(dev) for t in inputs], -1)
        for offset in (1, 16):
            source = torch.randn(3 * 64 * 64 + offset, generator=g).to(dtype)
            on_device = source.to(dev)
            cpu_view, dev_view = source[offset:].view(3, 64, 64), on_device[offset:].view(3, 64, 64)
            check([cpu_view] * 2, [dev_view] * 2, 1)
            check([cpu_view.transpose(0, 2)] * 2, [dev_view.transpose(0, 2)] * 2, 1)
        source = torch.randn(3, 64, 32, generator=g).to(dtype)
        on_device = source.to(dev)
        check(source.split(32, 1), on_device.split(32, 1), 1)
        check([source[:1].expand(3, -1, -1)] * 2, [on_device[:1].expand(3, -1, -1)] * 2, 1)
        empty = torch.empty(0, dtype=dtype)
        check([empty, source, empty], [empty.to(dev), on_device, empty.to(dev)], 1)
        check([empty, empty], [empty.to(dev), empty.to(dev)], 0)
        shaped_empty = torch.empty(3, 0, 32, dtype=dtype)
        check([shaped_empty, source], [shaped_empty.to(dev), on_device], 1)
        check([source], [on_device], 1)
        values = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), float("nan"), 1.0, -1.0, 0.5],
                              dtype=dtype).repeat(16)
        check([values, values], [values.to(dev), values.to(dev)], 0)
    assert cases[0] == 48


def _softmax_check(cpu, dev_tensor, dim, half_to_float=False):
    if half_to_float:
        actual = torch.ops.aten._softmax.default(dev_tensor, dim, True)
        expected = torch.softmax(cpu.float(), dim)
    else:
        actual = torch.softmax(dev_tensor, dim)
        expected = torch.softmax(cpu, dim)
    assert actual.device.type == "cuda"
    got = actual.cpu()
    assert got.dtype == expected.dtype and got.shape == expected.shape
    tol = 1e-3 if got.dtype == torch.float16 else 1e-5
    assert torch.equal(torch.isnan(got), torch.isnan(expected))
    assert torch.equal(torch.isposinf(got), torch.isposinf(expected))
    assert torch.equal(torch.isneginf(got), torch.isneginf(expected))
    finite = torch.isfinite(expected)
    err = (got.float()[finite] - expected.float()[finite]).abs().max().item() if finite.any() else 0.0
    assert err <= tol, (tuple(cpu.shape), dim, err)


def test_verify_softmax_checks(tb):
    """Softmax shapes and dims, large shifts, uniform rows, views, expands,
    coexistence with add/sigmoid/cat, non-finite rows, half_to_float
    (verify_softmax.py)."""
    dev = tb.device
    g = torch.Generator().manual_seed(2718)
    for dtype in (torch.float32, torch.float16):
        for shape, dims in (((), (0, -1)), ((0,), (0,)), ((2, 0, 3), (0, 1, 2)), ((1,), (0,)), ((3,), (0,)),
                            ((7,), (-1,)), ((100,), (0,)), ((3, 16), (-1, 0)), ((5, 1000), (1,)),
                            ((2, 2049), (1,)), ((2, 4097), (-1,)), ((2, 65537), (-1,)), ((2, 3, 7), (0, 1, 2, -2)),
                            ((2, 16, 17), (1,)), ((2, 1000, 17), (1,)), ((3, 7, 1), (1,)),
                            ((1, 4, 16, 8400), (1, 2)), ((1, 16, 4, 8400), (1,)), ((2, 4, 16, 2100), (2,))):
            cpu = (torch.randn(shape, generator=g) * 3).to(dtype)
            for dim in dims:
                _softmax_check(cpu, cpu.to(dev), dim)
        for shape, dim in (((3, 1000), -1), ((2, 16, 37), 1), ((2, 1000, 17), 1)):
            for shift in (-10000, 10000):
                cpu = (torch.randn(shape, generator=g) * 10 + shift).to(dtype)
                _softmax_check(cpu, cpu.to(dev), dim)
            cpu = torch.zeros(shape, dtype=dtype)
            _softmax_check(cpu, cpu.to(dev), dim)
        cpu = torch.randn(2, 3, 7, generator=g).to(dtype)
        d = cpu.to(dev)
        for dim in (0, 1, -1):
            _softmax_check(cpu.transpose(0, 2), d.transpose(0, 2), dim)
        _softmax_check(cpu[:, :, 1:6], d.as_strided((2, 3, 5), (21, 7, 1), 1), -1)
        _softmax_check(cpu[:, :, 1:6], d.as_strided((2, 3, 5), (21, 7, 1), 1), 1)
        _softmax_check(cpu.unsqueeze(0).expand(4, -1, -1, -1), d.unsqueeze(0).expand(4, -1, -1, -1), 0)
        for shape, dim in (((2, 16), -1), ((2, 16, 17), 1)):
            cpu = torch.randn(shape, generator=g).to(dtype)
            y = torch.softmax(cpu.to(dev), dim)
            ref = torch.softmax(cpu, dim)
            z = torch.cat((torch.add(y, y), torch.ops.thin_backend.sigmoid(y)), dim)
            expected = torch.cat((torch.add(ref, ref), torch.sigmoid(ref)), dim)
            tol = 1e-3 if dtype == torch.float16 else 1e-5
            assert (z.cpu().float() - expected.float()).abs().max().item() <= tol
        for values in ([float("-inf"), 0, 1], [float("-inf")] * 3, [0, float("inf"), 1], [0, float("nan"), 1]):
            a = torch.tensor(values, dtype=dtype)
            for shape, dim in (((1, 3), 1), ((3, 1), 0), ((3, 17), 0)):
                cpu = a.reshape((1, 3) if dim else (3, 1)).expand(shape).contiguous()
                _softmax_check(cpu, cpu.to(dev), dim)
        cpu = torch.tensor([[0, 0, float("-inf"), 0, 0], [1, float("nan"), float("-inf"), float("inf"), float("-inf")],
                            [2, 2, float("-inf"), 1, 3]], dtype=dtype)
        _softmax_check(cpu, cpu.to(dev), 0)
        _softmax_check(cpu.t().contiguous(), cpu.t().contiguous().to(dev), 1)
    for shape, dim in (((3, 1000), -1), ((2, 16, 17), 1)):
        cpu = torch.randn(shape, generator=g).half()
        _softmax_check(cpu, cpu.to(dev), dim, True)


def test_verify_graph_checks(tb):
    """CapturedForward: replay, call with a new input, shape check, owner thread,
    close twice, borrowed outputs outliving the graph, device-to-host rejected during
    capture (verify_graph.py)."""
    from thin_backend.graph import CapturedForward
    dev = tb.device

    def expression(x):
        return torch.sigmoid((x + x) * 0.5)

    x = torch.linspace(-2, 2, 2048).to(dev)
    graph = CapturedForward(expression, x)
    expected = expression(x).cpu()
    for _ in range(5):
        gc.collect()
        assert torch.equal(graph.replay().cpu(), expected)
    other = torch.linspace(1, 3, 2048).to(dev)
    assert torch.equal(graph(other).cpu(), expression(other).cpu())
    with pytest.raises(ValueError):
        graph(torch.empty(32, device=dev))
    errors = []

    def wrong_thread():
        for call in (graph.replay, lambda: graph(x)):
            try:
                call()
            except RuntimeError as error:
                errors.append(str(error))

    thread = threading.Thread(target=wrong_thread)
    thread.start()
    thread.join()
    assert len(errors) == 2 and all("creating thread/stream" in e for e in errors)
    second = CapturedForward(expression, x)
    retained = graph.outputs
    graph.close()
    graph.close()
    assert torch.equal(retained.cpu(), expression(other).cpu())
    assert torch.equal(second.replay().cpu(), expected)
    second.close()
    del graph, second
    gc.collect()
    assert torch.equal(expression(x).cpu(), expected)
    with pytest.raises(RuntimeError, match="Device-to-host"):
        CapturedForward(lambda value: value.cpu(), x)
    graph = CapturedForward(expression, x)
    assert torch.equal(graph.replay().cpu(), expected)
    retained = graph.outputs
    del graph
    gc.collect()
    assert torch.equal(retained.cpu(), expected)
