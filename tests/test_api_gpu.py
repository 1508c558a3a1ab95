"""GPU: the reference-facing API -- torch.ops namespaces, CapturedForward /
RuntimeGraph / FrozenGraph semantics (verify_graph.py), and ATen routing
(verify_ops.py, verify_all.py, verify_cat.py, verify_softmax.py call sites)."""
from __future__ import annotations

import threading

import pytest
import torch
import torch.nn.functional as F

from conftest import assert_bits_equal, ulp_diff
from oracle import ops as oops

pytestmark = pytest.mark.gpu


def test_thin_backend_ops(device):
    from thintnpu_b200 import library  # noqa: F401
    g = torch.Generator().manual_seed(42)
    for size in (5000, 65537, 1, 2047, 2048, 2049, 16385):
        a, b = torch.randn(size, generator=g), torch.randn(size, generator=g)
        assert_bits_equal(torch.ops.thin_backend.add(a.to(device), b.to(device)), a + b)
    for dtype in (torch.float32, torch.float16):
        a = torch.linspace(-8, 8, 65537, dtype=dtype)
        got = torch.ops.thin_backend.sigmoid(a.to(device)).cpu()
        if dtype == torch.float16:
            assert_bits_equal(got, torch.sigmoid(a))
        else:
            torch.testing.assert_close(got, torch.sigmoid(a), rtol=2e-6, atol=1e-7)
        for shape in ((1, 2, 5, 7), (2, 3, 13, 11), (1, 64, 80, 80)):
            x = torch.randn(shape, generator=g).to(dtype)
            assert_bits_equal(torch.ops.thin_backend.maxpool2d(x.to(device)), F.max_pool2d(x, 5, 1, 2))
            assert_bits_equal(torch.ops.thin_backend.upsample_nearest2d(x.to(device)),
                              F.interpolate(x, scale_factor=2, mode="nearest"))


def test_thin_native_flow_ops(device):
    from thintnpu_b200 import library  # noqa: F401
    g = torch.Generator().manual_seed(0)
    for c, h, w, k in ((256, 20, 20, 5), (32, 13, 17, 3), (16, 7, 9, 7), (48, 1, 31, 5)):
        xb = oops.to_blocked(torch.randn(1, c, h, w, generator=g).half())
        assert_bits_equal(torch.ops.thin_native_flow.maxpool(xb.to(device), k), oops.maxpool_blocked(xb, k))
    for c, h, w in ((128, 40, 40), (64, 13, 17), (16, 1, 33)):
        xb = oops.to_blocked(torch.randn(1, c, h, w, generator=g).half())
        assert_bits_equal(torch.ops.thin_native_flow.upsample(xb.to(device)), oops.upsample_blocked(xb))
    x = torch.randn(1, 64, 40, 40, generator=g).half()
    assert_bits_equal(torch.ops.thin_blocked.unpack(torch.ops.thin_blocked.pack(x.to(device))), x)


def test_captured_forward_semantics(device):
    from thintnpu_b200.graph import CapturedForward
    from thintnpu_b200.aten import aten_routing

    def expression(x):
        return torch.sigmoid((x + x) * 0.5)

    with torch.inference_mode(), aten_routing():
        x = torch.linspace(-2, 2, 2048, device=device)
        graph = CapturedForward(expression, x)
        expected = expression(x).cpu()
        for _ in range(5):
            assert torch.equal(graph.replay().cpu(), expected)
        other = torch.linspace(1, 3, 2048, device=device)
        assert torch.equal(graph(other).cpu(), expression(other).cpu())
        with pytest.raises(ValueError):
            graph(torch.empty(32, device=device))
        errors = []

        def wrong_thread():
            for call in (graph.replay, lambda: graph(x)):
                try:
                    call()
                except RuntimeError as error:
                    errors.append(str(error))
        t = threading.Thread(target=wrong_thread)
        t.start()
        t.join()
        assert len(errors) == 2 and all("creating thread/stream" in e for e in errors)
        second = CapturedForward(expression, x)
        retained = graph.outputs
        graph.close()
        graph.close()
        assert torch.equal(retained.cpu(), expression(other).cpu())
        assert torch.equal(second.replay().cpu(), expected)
        second.close()
        with pytest.raises(RuntimeError, match="Device-to-host"):
            CapturedForward(lambda value: value.cpu(), x)


def test_selection_capture_and_changed_input(device):
    from thintnpu_b200 import library  # noqa: F401
    from thintnpu_b200.graph import RuntimeGraph
    g = torch.Generator().manual_seed(3)
    base = torch.cat((torch.rand(2, 4, 8400, generator=g) * 640,
                      torch.randn(2, 80, 8400, generator=g).sigmoid()), 1).half().to(device)
    view = base.transpose(1, 2)
    with torch.inference_mode():
        eager = torch.ops.thin_native_flow.detection_select(view, 300, False)
        graph = RuntimeGraph()
        graph.begin()
        captured = torch.ops.thin_native_flow.detection_select(view, 300, False)
        graph.end()
        graph.replay()
        torch.cuda.synchronize()
        assert_bits_equal(captured, eager)
        base.neg_()
        changed = torch.ops.thin_native_flow.detection_select(view, 300, False)
        graph.replay()
        torch.cuda.synchronize()
        assert_bits_equal(captured, changed)
        graph.close()


def test_aten_routing_matches_cpu_and_routes(device):
    from thintnpu_b200 import aten
    g = torch.Generator().manual_seed(42)
    a = torch.randn(2, 7, 5, 7, generator=g).half()
    b = torch.randn(2, 7, 5, 7, generator=g).half() + 3
    before = dict(aten.ROUTED)
    with torch.inference_mode(), aten.aten_routing():
        x, y = a.to(device), b.to(device)
        assert_bits_equal(torch.cat((x, y, x), 1), torch.cat((a, b, a), 1))
        for op in ("add", "sub", "mul", "div"):
            assert_bits_equal(getattr(torch, op)(x, y), getattr(torch, op)(a, b))
        assert_bits_equal(x * 0.5, a * 0.5)
        assert_bits_equal(torch.sigmoid(x), torch.sigmoid(a))
        z = x.clone()
        F.silu(z, inplace=True)
        assert_bits_equal(z, F.silu(a))
        assert_bits_equal(F.silu(x), F.silu(a))
        s = torch.softmax(x, -1)
        assert (s.cpu().float() - torch.softmax(a, -1).float()).abs().max() <= 1e-3
        p = F.max_pool2d(x, 5, 1, 2)
        assert_bits_equal(p, F.max_pool2d(a.float(), 5, 1, 2).half())
        u = F.interpolate(x, scale_factor=2, mode="nearest")
        assert_bits_equal(u, F.interpolate(a.float(), scale_factor=2, mode="nearest").half())
        with pytest.raises(RuntimeError, match="k5/s1/p2"):
            F.max_pool2d(x, 3, 1, 1)
        # non-float work stays with PyTorch
        idx = torch.arange(10, device=device) + 1
        assert idx.sum().item() == 55
    with torch.inference_mode(), aten.aten_routing():
        v, i = F.max_pool2d(x, 5, 1, 2, return_indices=True)
        assert_bits_equal(v, p)
        assert int(i.abs().sum().item()) == 0  # zero placeholder indices (aten_adapter.cpp:69-80)
    for name in ("aten::cat", "aten::add", "aten::sigmoid", "aten::silu_", "aten::_softmax",
                 "aten::max_pool2d_with_indices", "aten::upsample_nearest2d"):
        assert aten.ROUTED.get(name, 0) > before.get(name, 0), name


def test_frozen_graph_region_contract(device):
    from thintnpu_b200.aten import aten_routing
    from thintnpu_b200.graph import FrozenGraph, RegionContract
    conv = torch.nn.Conv2d(16, 16, 1).half().to(device).requires_grad_(False).eval()

    def forward(x):
        return torch.sigmoid(x) + x

    with aten_routing():
        pilot = RegionContract([conv])
        x = torch.randn(1, 16, 8, 8, device=device).half()
        frozen = FrozenGraph(pilot, forward, x)
        out = frozen.replay().clone()
        assert_bits_equal(out, forward(x))
        assert_bits_equal(frozen(x * 2).clone(), forward(x * 2))
        with torch.no_grad():
            conv.weight.add_(1)
        with pytest.raises(ValueError, match="version or gradient mode changed"):
            frozen.replay()
        frozen.close()


def _contract_breakers():
    """(description, mutation, expected message) for RegionContract.validate."""
    def replace_weight(m):
        m.weight = torch.nn.Parameter(m.weight.detach().clone(), requires_grad=False)

    def hook(m):
        m.register_forward_hook(lambda *a: None)

    def rebind(m):
        m.forward = lambda x: x

    def add_child(m):
        m.extra = torch.nn.Identity()

    return [("in-place update", lambda m: m.weight.mul_(1), "version or gradient mode changed"),
            ("replaced parameter", replace_weight, "identity changed"),
            ("stride", lambda m: setattr(m, "stride", (2, 2)), "operator configuration changed"),
            ("training mode", lambda m: m.train(), "inference-only"),
            ("forward hook", hook, "hooks changed"),
            ("rebound forward", rebind, "forward changed"),
            ("new child", add_child, "children changed")]


@pytest.mark.parametrize("case", range(7))
def test_region_contract_detects_each_change(device, case):
    from thintnpu_b200.graph import RegionContract
    name, mutate, message = _contract_breakers()[case]
    conv = torch.nn.Conv2d(16, 16, 3, padding=1).half().to(device).requires_grad_(False).eval()
    pilot = RegionContract([torch.nn.Sequential(conv).eval()])
    pilot.validate()
    with torch.no_grad():
        mutate(conv)
    with pytest.raises(ValueError, match=message):
        pilot.validate()


def test_region_contract_rejects_unprepared_parameters(device):
    from thintnpu_b200.graph import RegionContract
    with pytest.raises(ValueError, match="FP16 CUDA inference"):
        RegionContract([torch.nn.Conv2d(16, 16, 1).half().to(device)])  # requires_grad
    with torch.inference_mode():
        inference = torch.nn.Conv2d(16, 16, 1).half().to(device)
    with pytest.raises(ValueError, match="no_grad"):
        RegionContract([inference])


def test_bias_silu_residual_via_torch_ops(device):
    from thintnpu_b200 import library  # noqa: F401
    g = torch.Generator().manual_seed(1)
    x = oops.to_blocked(torch.randn(2, 64, 20, 20, generator=g).half())
    r = oops.to_blocked(torch.randn(2, 64, 20, 20, generator=g).half())
    b = (torch.randn(64, generator=g) * 0.1).half()
    got = torch.ops.thin_native_flow.bias_silu_residual(x.to(device), b.to(device), r.to(device))
    assert ulp_diff(got, oops.bias_silu_residual(x, b, r)).max() <= 2


def test_memory_entry_points_round_trip(device):
    """ttn_malloc / ttn_malloc_host / ttn_memcpy_async / ttn_free*: host -> device ->
    device -> host through the C ABI returns the bytes; 0 bytes gives a null pointer;
    freeing null is a no-op; an unknown copy kind is refused."""
    import ctypes
    from thintnpu_b200 import _lib
    lib = _lib.lib()
    n = 1000003  # not a multiple of the 32-byte block
    ptrs = [ctypes.c_void_p() for _ in range(4)]
    host_in, dev_a, dev_b, host_out = ptrs
    _lib.check("ttn_malloc_host", lib.ttn_malloc_host(ctypes.byref(host_in), n))
    _lib.check("ttn_malloc_host", lib.ttn_malloc_host(ctypes.byref(host_out), n))
    _lib.check("ttn_malloc", lib.ttn_malloc(ctypes.byref(dev_a), n))
    _lib.check("ttn_malloc", lib.ttn_malloc(ctypes.byref(dev_b), n))
    assert all(p.value for p in ptrs) and dev_a.value % 256 == 0
    pattern = bytes((i * 7 + 3) & 0xFF for i in range(n))
    ctypes.memmove(host_in.value, pattern, n)
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check("ttn_memcpy_async", lib.ttn_memcpy_async(dev_a, host_in, n, 0, stream))
    _lib.check("ttn_memcpy_async", lib.ttn_memcpy_async(dev_b, dev_a, n, 2, stream))
    _lib.check("ttn_memcpy_async", lib.ttn_memcpy_async(host_out, dev_b, n, 1, stream))
    torch.cuda.synchronize(device)
    assert ctypes.string_at(host_out.value, n) == pattern
    assert lib.ttn_memcpy_async(dev_b, dev_a, n, 7, stream) == 1  # TTN_INVALID_ARG
    zero = ctypes.c_void_p(123)
    _lib.check("ttn_malloc", lib.ttn_malloc(ctypes.byref(zero), 0))
    assert zero.value is None
    assert lib.ttn_free(None) == 0 and lib.ttn_free_host(None) == 0
    for p, free in ((dev_a, lib.ttn_free), (dev_b, lib.ttn_free), (host_in, lib.ttn_free_host),
                    (host_out, lib.ttn_free_host)):
        _lib.check("ttn_free", free(p))
