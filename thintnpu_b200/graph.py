"""Frozen-graph replay on CUDA Graphs, mirroring the reference's graph API.

* ``RuntimeGraph`` -- begin/end/replay/close with the owner-thread and state
  checks of thin_backend::RuntimeGraph (backend.cpp:62-113).  Capture runs on a
  side stream in thread-local capture mode; tensors allocated during capture come
  from the graph's private memory pool and stay valid while referenced.
  Device-to-host copies are rejected while capturing (ops.cpp:40).
* ``CapturedForward`` -- fixed-shape inference with a static input and borrowed
  outputs (thin_backend/graph.py:6-51): three warm-ups, capture, replay;
  ``__call__`` validates shape/dtype/device/layout/strides and the thread.
* ``RegionContract`` / ``FrozenGraph`` -- replay only while the captured modules'
  parameters, buffers and structural attributes are unchanged
  (region_contract.py, blocked_graph.py:4-23), checked in Python.
"""
from __future__ import annotations

from threading import get_ident
from typing import Iterable, Optional

import torch
from torch.utils._python_dispatch import TorchDispatchMode

OWNER_ERROR = "RuntimeGraph must stay on its creating thread/stream"


class _RejectDeviceToHost(TorchDispatchMode):
    """Raises on any copy that would read CUDA memory into host memory."""

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        name = func.overloadpacket.__name__
        if name in ("_to_copy", "to", "copy_", "_copy_from", "_copy_from_and_resize"):
            src = args[1] if name == "copy_" else args[0]
            dst_device = kwargs.get("device")
            if name == "copy_":
                dst_device = args[0].device
            if (isinstance(src, torch.Tensor) and src.is_cuda and dst_device is not None
                    and torch.device(dst_device).type == "cpu"):
                raise RuntimeError("Device-to-host copy is not allowed during graph capture")
        if name == "_local_scalar_dense":
            raise RuntimeError("Device-to-host copy is not allowed during graph capture")
        return func(*args, **kwargs)


class RuntimeGraph:
    """CUDA-graph capture of the current thread's work (thin_backend::RuntimeGraph)."""

    def __init__(self):
        self._owner = get_ident()
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self._stream: Optional[torch.cuda.Stream] = None
        self._stream_ctx = None
        self._guard = None
        self._active = False
        self._closed = False
        self._captured = False

    def _same_thread(self):
        if get_ident() != self._owner:
            raise RuntimeError(OWNER_ERROR)

    def begin(self):
        self._same_thread()
        if self._closed or self._active or self._captured or torch.cuda.is_current_stream_capturing():
            raise RuntimeError("RuntimeGraph cannot begin in its current state")
        current = torch.cuda.current_stream()
        self._stream = torch.cuda.Stream()
        self._stream.wait_stream(current)
        self._graph = torch.cuda.CUDAGraph()
        self._stream_ctx = torch.cuda.stream(self._stream)
        self._stream_ctx.__enter__()
        try:
            self._graph.capture_begin(capture_error_mode="thread_local")
        except Exception:
            self._stream_ctx.__exit__(None, None, None)
            raise
        self._guard = _RejectDeviceToHost()
        self._guard.__enter__()
        self._active = True

    def end(self):
        self._same_thread()
        if not self._active:
            raise RuntimeError("RuntimeGraph is not capturing")
        self._active = False
        try:
            self._guard.__exit__(None, None, None)
            self._graph.capture_end()
        finally:
            self._stream_ctx.__exit__(None, None, None)
            torch.cuda.current_stream().wait_stream(self._stream)
        self._captured = True

    def replay(self):
        self._same_thread()
        if self._closed or not self._captured or self._active or torch.cuda.is_current_stream_capturing():
            raise RuntimeError("RuntimeGraph is not ready to replay")
        self._graph.replay()

    def close(self):
        self._same_thread()
        if self._closed:
            return
        if self._active:
            try:
                self.end()
            except Exception:
                pass
        torch.cuda.synchronize()
        self._graph = None
        self._closed = True


class CapturedForward:
    """Fixed-shape inference with graph-owned workspace and borrowed output buffers.

    The callable, its parameters and captured tensors must not be mutated or moved.
    Calls reuse the returned output tensors; clone outputs to retain prior results.
    Create, replay and close on the same thread.  No concurrent replay is supported."""

    def __init__(self, forward, example: torch.Tensor, warmup: int = 3):
        if not example.is_cuda or example.requires_grad:
            raise ValueError("CapturedForward requires an inference-only CUDA input")
        self._input_layout = example.layout
        self._input_stride = example.stride()
        self._thread = get_ident()
        self.forward = forward
        self.input = torch.empty_like(example)
        self.input.copy_(example)
        self.outputs = None
        self.graph = RuntimeGraph()
        with torch.inference_mode():
            for _ in range(warmup):
                forward(self.input)
            torch.cuda.synchronize()
            self.graph.begin()
            try:
                self.outputs = forward(self.input)
            finally:
                self.graph.end()
        self.graph.replay()

    def replay(self):
        """Enqueue one replay using the existing static input; return borrowed outputs."""
        self.graph.replay()
        return self.outputs

    def __call__(self, value: torch.Tensor):
        if get_ident() != self._thread:
            raise RuntimeError(OWNER_ERROR)
        if (value.shape != self.input.shape or value.dtype != self.input.dtype
                or value.device != self.input.device or value.requires_grad
                or value.layout != self._input_layout or value.stride() != self._input_stride):
            raise ValueError("Graph input shape, dtype, device and layout/strides must match capture")
        self.input.copy_(value)
        return self.replay()

    def close(self):
        self.graph.close()


class RegionContract:
    """Guards a captured region: modules' parameters/buffers (identity, version,
    storage, shape, dtype, device) and listed structural attributes must not change
    between capture and replay (the contract of region_contract.py)."""

    attributes = ("in_channels", "out_channels", "kernel_size", "stride", "padding", "dilation",
                  "groups", "add", "c", "inplace", "scale_factor", "mode", "size", "ceil_mode",
                  "num_heads", "head_dim", "key_dim", "scale", "shortcut", "n", "nl", "na", "no",
                  "nc", "export", "reg_max", "end2end", "max_det", "agnostic_nms", "xyxy")

    def __init__(self, roots: Iterable[torch.nn.Module]):
        self.modules = tuple(m for root in roots for m in root.modules())
        for module in self.modules:
            for tensor in (*module._parameters.values(), *module._buffers.values()):
                if tensor is None:
                    continue
                try:
                    tensor._version
                except RuntimeError as error:
                    raise ValueError("Prepare versioned parameters under no_grad(), not inference_mode()") \
                        from error
                if tensor.requires_grad or tensor.dtype != torch.float16 or not tensor.is_cuda:
                    raise ValueError("Expected fixed FP16 CUDA inference parameters")
        self._snapshot = self._state()

    def _state(self):
        state = []
        for module in self.modules:
            tensors = tuple((name, id(t), t._version, t.data_ptr(), tuple(t.shape), t.dtype, t.device)
                            for name, t in (*module._parameters.items(), *module._buffers.items())
                            if t is not None)
            attrs = tuple((a, repr(getattr(module, a))) for a in self.attributes if hasattr(module, a))
            state.append((id(module), type(module), module.training, tensors, attrs))
        return tuple(state)

    def validate(self):
        if self._state() != self._snapshot:
            raise RuntimeError("Frozen region changed since capture (parameters, buffers or attributes)")


class FrozenGraph:
    """CapturedForward replayed only while the pilot's region contract holds
    (blocked_graph.py:4-23)."""

    def __init__(self, pilot, forward, example):
        pilot.validate()
        self.pilot = pilot
        self.graph = CapturedForward(forward, example)

    @property
    def outputs(self):
        return self.graph.outputs

    def replay(self):
        self.pilot.validate()
        return self.graph.replay()

    def __call__(self, value):
        self.pilot.validate()
        return self.graph(value)

    def close(self):
        self.graph.close()
