"""CPU: the reference's operator schemas are registered with Meta kernels
(verify_all.py:117-126 checks the same dispatch keys)."""
from __future__ import annotations

import torch

from thintnpu_b200 import library  # noqa: F401


def test_schemas_and_dispatch_keys():
    for op in ("add", "sigmoid", "maxpool2d", "upsample_nearest2d"):
        for key in ("CUDA", "AutogradCUDA", "Meta"):
            assert torch._C._dispatch_has_kernel_for_dispatch_key("thin_backend::" + op, key), (op, key)
    for op in ("maxpool", "upsample", "detection_select", "detection_select_trace", "silu_", "sppf",
               "softmax", "dfl_decode", "bias_silu_residual", "conv", "depthwise", "pack_input"):
        for key in ("CUDA", "AutogradCUDA", "Meta"):
            assert torch._C._dispatch_has_kernel_for_dispatch_key("thin_native_flow::" + op, key), (op, key)
    for op in ("pack", "unpack", "conv"):
        assert torch._C._dispatch_has_kernel_for_dispatch_key("thin_blocked::" + op, "Meta"), op


def test_meta_shapes():
    meta = lambda *s, dtype=torch.float16: torch.empty(*s, device="meta", dtype=dtype)
    assert torch.ops.thin_backend.add(meta(5000, dtype=torch.float32), meta(5000, dtype=torch.float32)).shape == (5000,)
    assert torch.ops.thin_backend.sigmoid(meta(65537)).device.type == "meta"
    assert torch.ops.thin_backend.maxpool2d(meta(1, 16, 8, 8)).shape == (1, 16, 8, 8)
    assert torch.ops.thin_backend.upsample_nearest2d(meta(1, 16, 8, 8)).shape == (1, 16, 16, 16)
    assert torch.ops.thin_native_flow.upsample(meta(2, 3, 5, 7, 16)).shape == (2, 3, 10, 14, 16)
    assert torch.ops.thin_native_flow.sppf(meta(2, 16, 20, 20, 16)).shape == (2, 64, 20, 20, 16)
    out = torch.ops.thin_native_flow.detection_select(meta(2, 8400, 84), 300, False)
    assert out.shape == (2, 300, 6) and out.dtype == torch.float32
    trace = torch.ops.thin_native_flow.detection_select_trace(meta(2, 8400, 84), 300, True)
    assert [tuple(t.shape) for t in trace] == [(2, 300, 6), (2, 8400), (2, 300), (2, 0, 80), (2, 300),
                                               (2, 0), (2, 300), (2, 300)]
    assert torch.ops.thin_blocked.pack(meta(1, 40, 5, 7)).shape == (1, 3, 5, 7, 16)
    assert torch.ops.thin_blocked.unpack(meta(1, 3, 5, 7, 16)).shape == (1, 48, 5, 7)
    dec = torch.ops.thin_native_flow.dfl_decode(meta(2, 64, 8400), meta(2, 80, 8400), [80, 40, 20],
                                                [80, 40, 20], [8.0, 16.0, 32.0])
    assert dec.shape == (2, 84, 8400)
    nf, bl = torch.ops.thin_native_flow, torch.ops.thin_blocked
    x = meta(2, 8, 40, 40, 16)
    assert nf.conv(x, meta(8, 9, 128, 16), meta(128), 128, 3, 2).shape == (2, 8, 20, 20, 16)
    assert nf.conv(x, meta(8, 1, 128, 16), None, 80, 1, 1, False, True).shape == (2, 80, 40, 40)
    assert nf.depthwise(x, meta(8, 3, 3, 16), meta(128), 3, 1).shape == (2, 8, 40, 40, 16)
    assert nf.depthwise(x, meta(8, 5, 5, 16), None, 5, 2).shape == (2, 8, 20, 20, 16)
    assert bl.conv(x, meta(8, 1, 256, 16), meta(256), 256, 1, 1, False, True).shape == (2, 16, 40, 40, 16)
    assert nf.pack_input(meta(1, 3, 64, 64)).shape == (1, 1, 64, 64, 16)


def test_import_thin_backend_registers_and_routes():
    """``import thin_backend`` registers the namespaces and loads the library like the
    reference's import; ATen routing stays off unless THIN_BACKEND_ATEN=1."""
    import subprocess
    import sys
    code = ("import torch, thin_backend\n"
            "from thintnpu_b200 import aten\n"
            "assert thin_backend.device == 'cuda'\n"
            "import os\n"
            "assert (aten._GLOBAL is not None) == (os.environ.get('THIN_BACKEND_ATEN') == '1')\n"
            "assert torch._C._dispatch_has_kernel_for_dispatch_key('thin_native_flow::detection_select', 'CUDA')\n"
            "from thin_backend.graph import CapturedForward\n"
            "from thin_backend.blocked_graph import FrozenGraph\n"
            "print('ok')\n")
    import os
    from conftest import ROOT
    for flag in ("0", "1"):
        env = dict(os.environ, THIN_BACKEND_ATEN=flag)
        done = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300,
                              env=env)
        assert done.returncode == 0 and "ok" in done.stdout, done.stderr
