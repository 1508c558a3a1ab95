"""Frozen-graph replay on CUDA Graphs, mirroring the reference's graph API.

* ``RuntimeGraph`` -- begin/end/replay/close with the owner-thread and state
  checks of thin_backend::RuntimeGraph (backend.cpp:62-113).  Capture runs on a
  side stream in thread-local capture mode; tensors allocated during capture come
  from the graph's private memory pool and stay valid while referenced.
  Device-to-host copies are rejected while capturing (ops.cpp:40).
* ``CapturedForward`` -- fixed-shape inference as one CUDA graph with a
  graph-owned static input and borrowed outputs (the interface of
  thin_backend/graph.py:6-51: ``replay()``, ``__call__(x)``, ``close()``,
  ``outputs``); the input's signature is checked on every call.
* ``RegionContract`` / ``FrozenGraph`` -- replay only while the captured
  modules are as they were at capture (the interface of region_contract.py and
  blocked_graph.py:4-23): a per-tensor version vector plus identity and
  configuration records, compared once per replay.
"""
from __future__ import annotations

from dataclasses import dataclass
from threading import get_ident
from typing import Iterable, Optional, Tuple

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


@dataclass(frozen=True)
class _InputSignature:
    """What a replay input must share with the captured one."""
    shape: Tuple[int, ...]
    stride: Tuple[int, ...]
    dtype: torch.dtype
    device: torch.device
    layout: torch.layout

    @classmethod
    def of(cls, t: torch.Tensor) -> "_InputSignature":
        return cls(tuple(t.shape), tuple(t.stride()), t.dtype, t.device, t.layout)

    def admits(self, t: torch.Tensor) -> bool:
        return isinstance(t, torch.Tensor) and not t.requires_grad and _InputSignature.of(t) == self


def _record(forward, static_input: torch.Tensor, warmup: int):
    """Runs `forward` `warmup` times on a side stream (so the caching allocator
    settles before capture), then captures one call; returns (graph, outputs)."""
    current = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    side.wait_stream(current)
    with torch.inference_mode():
        with torch.cuda.stream(side):
            for _ in range(warmup):
                forward(static_input)
        current.wait_stream(side)
        graph = RuntimeGraph()
        graph.begin()
        try:
            outputs = forward(static_input)
        finally:
            graph.end()
    return graph, outputs


class CapturedForward:
    """``forward(input)`` frozen into one CUDA graph for a fixed input signature.

    The graph owns a static copy of the input (same strides) and returns the
    tensors ``forward`` produced during capture as its outputs: they are borrowed,
    and every replay overwrites them in place (clone what must survive).  The
    callable and the tensors it captured must stay unmodified and in place.  Use
    from the creating thread only, one replay at a time."""

    def __init__(self, forward, example: torch.Tensor, warmup: int = 3):
        if not (isinstance(example, torch.Tensor) and example.is_cuda) or example.requires_grad:
            raise ValueError("CapturedForward requires an inference-only CUDA input")
        self._signature = _InputSignature.of(example)
        self._owner = get_ident()
        self.forward = forward
        self.input = torch.empty_strided(example.size(), example.stride(), dtype=example.dtype,
                                         device=example.device)
        self.input.copy_(example)
        self.graph, self.outputs = _record(forward, self.input, warmup)
        self.graph.replay()

    def _check_caller(self) -> None:
        if get_ident() != self._owner:
            raise RuntimeError(OWNER_ERROR)

    def _run(self, value: Optional[torch.Tensor]):
        self._check_caller()
        if value is not None:
            if not self._signature.admits(value):
                raise ValueError("Graph input shape, dtype, device and layout/strides must match capture")
            self.input.copy_(value)
        self.graph.replay()
        return self.outputs

    def replay(self):
        """Enqueue one replay on the static input as it stands; returns the borrowed outputs."""
        return self._run(None)

    def __call__(self, value: torch.Tensor):
        """Copy `value` into the static input, replay, return the borrowed outputs."""
        return self._run(value)

    def close(self):
        self.graph.close()


_TENSOR_GROUPS = ("_parameters", "_buffers")
_CHANGED = "Region parameter/prepack version or gradient mode changed"


class RegionContract:
    """Capture-time contract of a region of modules, checked before each replay.

    At construction every parameter and buffer must be a fixed fp16 CUDA
    inference tensor.  Recorded then, and compared by ``validate``:

    * a version vector -- the autograd version counter of every parameter and
      buffer of the region, in one flat list (an in-place update bumps it);
    * per module: its class, training flag, children, hooks, forward binding
      (unless the module is in ``ignored_forward``), the listed configuration
      attributes, and for each tensor slot the tensor object and its storage
      (pointer, offset, sizes, strides, dtype, device, requires_grad).

    ``validate`` raises ValueError naming what changed."""

    attributes = ("in_channels", "out_channels", "kernel_size", "stride", "padding", "padding_mode",
                  "dilation", "groups", "add", "c", "inplace", "scale_factor", "mode", "align_corners",
                  "size", "ceil_mode", "return_indices", "num_heads", "head_dim", "key_dim", "scale",
                  "shortcut", "n", "_thin_attention_prescale", "nl", "na", "no", "nc", "export", "reg_max",
                  "end2end", "_thin_strides", "max_det", "agnostic_nms", "xyxy")

    def __init__(self, roots: Iterable[torch.nn.Module], ignored_forward=()):
        self.modules = tuple(m for root in roots for m in root.modules())
        ignored = set(id(m) for m in ignored_forward)
        self._tensors = []   # flat, in record order
        self._records = []
        for module in self.modules:
            slots = []
            for group in _TENSOR_GROUPS:
                for name, t in getattr(module, group).items():
                    if t is not None:
                        _check_inference_tensor(t)
                        self._tensors.append(t)
                    slots.append((group, name, t, _storage_key(t)))
            forward = None if id(module) in ignored else module.__dict__.get("forward")
            self._records.append((module, type(module), tuple(slots), _children(module), forward,
                                  id(module) in ignored, _configuration(module, self.attributes)))
        self._versions = [t._version for t in self._tensors]

    def validate(self):
        if any(module.training for module in self.modules):
            raise ValueError("Region is inference-only")
        if _global_hooks():
            raise ValueError("Global module hooks are unsupported")
        if [t._version for t in self._tensors] != self._versions:
            raise ValueError(_CHANGED)
        for module, cls, slots, children, forward, ignored, config in self._records:
            if type(module) is not cls:
                raise ValueError("Region module class changed")
            if _hooked(module):
                raise ValueError("Region hooks changed")
            now = _children(module)
            if len(now) != len(children) or any(a[0] != b[0] for a, b in zip(now, children)):
                raise ValueError("Region children changed")
            if any(a[1] is not b[1] for a, b in zip(now, children)):
                raise ValueError("Region child identity changed")
            if not ignored and module.__dict__.get("forward") is not forward:
                raise ValueError("Region forward changed")
            for name, value in config:
                if not hasattr(module, name):
                    raise ValueError("Region attribute removed")
                current = getattr(module, name)
                if current is not value and current != value:
                    raise ValueError("Region operator configuration changed")
            count = sum(len(getattr(module, group)) for group in _TENSOR_GROUPS)
            if count != len(slots):
                raise ValueError("Region parameter/buffer set changed")
            for group, name, t, key in slots:
                if getattr(module, group).get(name, _MISSING) is not t:
                    raise ValueError("Region parameter/prepack identity changed")
                if t is not None and _storage_key(t) != key:
                    raise ValueError(_CHANGED)


_MISSING = object()


def _check_inference_tensor(t: torch.Tensor) -> None:
    try:
        t._version
    except RuntimeError as error:  # inference tensors carry no version counter
        raise ValueError("Prepare versioned parameters under no_grad(), not inference_mode()") from error
    if t.requires_grad or t.dtype != torch.float16 or not t.is_cuda:
        raise ValueError("Expected fixed FP16 CUDA inference parameters")


def _storage_key(t):
    if t is None:
        return None
    return (t.data_ptr(), t.storage_offset(), tuple(t.shape), tuple(t.stride()), t.dtype, t.device,
            t.requires_grad)


def _children(module):
    return tuple(module._modules.items())


def _configuration(module, names):
    return tuple((name, getattr(module, name)) for name in names if hasattr(module, name))


def _hooked(module) -> bool:
    return bool(module._forward_hooks or module._forward_pre_hooks)


def _global_hooks() -> bool:
    from torch.nn.modules import module as nn_module
    return bool(nn_module._global_forward_hooks or nn_module._global_forward_pre_hooks)


class FrozenGraph(CapturedForward):
    """A CapturedForward that replays only while `pilot` (a RegionContract over
    the modules `forward` uses) still validates: checked before capture and
    before every replay."""

    def __init__(self, pilot, forward, example):
        pilot.validate()
        self.pilot = pilot
        super().__init__(forward, example)

    def _run(self, value):
        self.pilot.validate()
        return super()._run(value)
