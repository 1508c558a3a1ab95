"""ThinTNPU-B200: the fp16 op pass between YOLO convolutions as sm_100a CUDA kernels.

``libttn.so`` (include/ttn.h) is the product: hand-written kernels behind a
C ABI.  This package binds it with ctypes and exposes the reference's
``thin_backend`` operator surface on CUDA tensors.  The library loads on the
first op call (or ``load()``) and a missing library raises ImportError -- there
is no CPU or PyTorch fallback.
"""
from . import _lib
from . import ops  # noqa: E402
from .ops import (add, add_silu, attention, bias_silu_residual, cat, contiguous, conv2d, conv2d_pack_weights,
                  copy_, depthwise, depthwise_pack_weights, detection_select,  # noqa: E402,F401
                  dfl_decode, div, maxpool2d, maxpool_blocked, mul, pack, sigmoid, silu, silu_,
                  softmax, sppf, sub, unpack, upsample_blocked, upsample_nearest2d)

__version__ = "0.1.0"


def load():
    """Load libttn.so now (raises ImportError when it is missing or stale)."""
    return _lib.lib()
