"""Drop-in import path for code written against the reference's ``thin_backend``.

``import thin_backend`` registers the operator namespaces
(``torch.ops.thin_backend``, ``torch.ops.thin_native_flow``,
``torch.ops.thin_blocked``) backed by libttn on CUDA tensors and, like the
reference's import side effect (thin_backend/__init__.py:5-18), routes the op
pass's ATen calls on CUDA float tensors to libttn for the rest of the process
(set ``THIN_BACKEND_ATEN=0`` to keep PyTorch's own kernels).  The device is
``cuda`` (the reference's ``npu``).
"""
import os

import thintnpu_b200
from thintnpu_b200 import library as _library  # noqa: F401  (registers torch.ops namespaces)
from thintnpu_b200.aten import aten_routing, disable_aten_routing, enable_aten_routing  # noqa: F401
from thintnpu_b200.graph import CapturedForward, RuntimeGraph  # noqa: F401

device = "cuda"

thintnpu_b200.load()
if os.environ.get("THIN_BACKEND_ATEN", "1") != "0":
    enable_aten_routing()
