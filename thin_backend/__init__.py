"""Drop-in import path for code written against the reference's ``thin_backend``.

``import thin_backend`` registers the operator namespaces
(``torch.ops.thin_backend``, ``torch.ops.thin_native_flow``,
``torch.ops.thin_blocked``) backed by libttn on CUDA tensors and loads the
library (thin_backend/__init__.py:5-18 registers the reference's device the
same way).  The reference's ``npu`` device is ``cuda`` here (``device``): a
script written for the reference runs with ``.to('npu')`` replaced by
``.to(thin_backend.device)``.

The reference also routes ATen calls on its own device to its kernels.  CUDA
tensors are PyTorch's as well, so that routing is opt-in here:
``with thin_backend.aten_routing(): ...`` for a block, ``enable_aten_routing()``
for the rest of the process, or ``THIN_BACKEND_ATEN=1`` in the environment to
turn it on at import.
"""
import os

import thintnpu_b200
from thintnpu_b200 import library as _library  # noqa: F401  (registers torch.ops namespaces)
from thintnpu_b200.aten import aten_routing, disable_aten_routing, enable_aten_routing  # noqa: F401
from thintnpu_b200.graph import CapturedForward, RuntimeGraph  # noqa: F401

device = "cuda"

thintnpu_b200.load()
if os.environ.get("THIN_BACKEND_ATEN", "0") == "1":
    enable_aten_routing()
