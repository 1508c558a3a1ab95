"""The YOLOv8s-640 non-conv op pass as a static plan, and its CUDA executor.

Every convolution output is an input of the pass (seeded N(0,1) data at the
conv's true NC1HWC0 shape); the pass runs everything between the convs, in
model order:

* SiLU on each of the 57 activated conv outputs (conv_flow.cpp:57-84 fuses it
  into the conv epilogue in the reference; here it is its own kernel),
* C2f ``chunk(2, 1)`` as channel-block views and the Bottleneck residual adds,
* the C2f / neck concats along C1 (ops.cpp:419-462),
* SPPF: three chained 5x5 max-pools and their concat (flow_ops.cpp:208-231),
* two nearest-2x upsamples (flow_ops.cpp:233-252),
* the Detect-terminal NC1HWC0 -> NCHW restore into one [B, 144, 8400] head
  (conv_flow.cpp:87-121, anchorfree_predictions whole_blocked.py:118-135),
* the DFL / anchor decode with sigmoid scores (whole_blocked.py:136-146).

Topology: Ultralytics yolov8s (depth 0.33, width 0.50, max 1024 channels),
restated from the published model definition; channel widths 32/64/128/256/512.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import ops

C0 = 16


@dataclass(frozen=True)
class Ref:
    """A channel-block slice [start, start+count) of a named NC1HWC0 tensor."""
    name: str
    start: int
    count: int


@dataclass(frozen=True)
class Step:
    op: str                      # silu | add | cat | sppf | upsample | restore | decode
    inputs: Tuple[Ref, ...]
    output: Optional[str]
    attrs: Tuple = ()


@dataclass
class Plan:
    imgsz: int
    nc: int
    shapes: Dict[str, Tuple[int, int, int]] = field(default_factory=dict)  # name -> (c1, h, w)
    conv_inputs: List[str] = field(default_factory=list)  # synthetic pass inputs, in model order
    # per conv (same order): its input (None = the image) and (kernel, stride)
    conv_sources: List[Optional[Ref]] = field(default_factory=list)
    conv_kernels: List[Tuple[int, int]] = field(default_factory=list)
    steps: List[Step] = field(default_factory=list)
    # the model order of convs and steps: ("conv", conv index) / ("step", step index)
    order: List[Tuple[str, int]] = field(default_factory=list)
    levels: List[Tuple[int, int]] = field(default_factory=list)
    strides: List[float] = field(default_factory=list)

    @property
    def anchors(self) -> int:
        return sum(h * w for h, w in self.levels)

    def elements(self, name: str) -> int:
        c1, h, w = self.shapes[name]
        return c1 * h * w * C0

    def step_bytes(self, step: Step) -> int:
        """Compulsory bytes of one step for one image (inputs read + output written)."""
        def ref_elems(r: Ref) -> int:
            _, h, w = self.shapes[r.name]
            return r.count * h * w * C0
        if step.op == "silu":
            return 2 * 2 * ref_elems(step.inputs[0])
        if step.op == "add":
            return 3 * 2 * ref_elems(step.inputs[0])
        if step.op == "cat":
            return 2 * 2 * sum(ref_elems(r) for r in step.inputs)
        if step.op == "sppf":
            return 2 * (1 + 4) * ref_elems(step.inputs[0])
        if step.op == "upsample":
            return 2 * (1 + 4) * ref_elems(step.inputs[0])
        if step.op == "restore":
            channels = step.attrs[1]
            _, h, w = self.shapes[step.inputs[0].name]
            return 2 * 2 * channels * h * w
        if step.op == "decode":
            return 2 * (64 + self.nc + 4 + self.nc) * self.anchors
        raise ValueError(step.op)

    def bytes_per_image(self) -> Dict[str, int]:
        out: Dict[str, int] = {}
        for s in self.steps:
            out[s.op] = out.get(s.op, 0) + self.step_bytes(s)
        return out


class _Builder:
    def __init__(self, imgsz: int, nc: int):
        self.plan = Plan(imgsz=imgsz, nc=nc)
        self.count = 0

    def _new(self, prefix: str, c1: int, h: int, w: int) -> str:
        name = f"{prefix}{self.count}"
        self.count += 1
        self.plan.shapes[name] = (c1, h, w)
        return name

    def step(self, step: Step) -> None:
        self.plan.order.append(("step", len(self.plan.steps)))
        self.plan.steps.append(step)

    def conv(self, channels: int, h: int, w: int, act: bool = True, src: Optional[Ref] = None,
             k: int = 1, s: int = 1) -> Ref:
        """A conv with `channels` outputs at h x w from `src` (None: the image)."""
        c1 = (channels + C0 - 1) // C0
        raw = self._new("conv", c1, h, w)
        self.plan.order.append(("conv", len(self.plan.conv_inputs)))
        self.plan.conv_inputs.append(raw)
        self.plan.conv_sources.append(src)
        self.plan.conv_kernels.append((k, s))
        if not act:
            return Ref(raw, 0, c1)
        out = self._new("act", c1, h, w)
        self.step(Step("silu", (Ref(raw, 0, c1),), out))
        return Ref(out, 0, c1)

    def add(self, a: Ref, b: Ref) -> Ref:
        _, h, w = self.plan.shapes[a.name]
        out = self._new("add", a.count, h, w)
        self.step(Step("add", (a, b), out))
        return Ref(out, 0, a.count)

    def cat(self, refs: Sequence[Ref]) -> Ref:
        _, h, w = self.plan.shapes[refs[0].name]
        total = sum(r.count for r in refs)
        out = self._new("cat", total, h, w)
        self.step(Step("cat", tuple(refs), out))
        return Ref(out, 0, total)

    def upsample(self, x: Ref) -> Ref:
        _, h, w = self.plan.shapes[x.name]
        out = self._new("up", x.count, 2 * h, 2 * w)
        self.step(Step("upsample", (x,), out))
        return Ref(out, 0, x.count)

    def sppf_pools(self, x: Ref, k: int = 5) -> Ref:
        _, h, w = self.plan.shapes[x.name]
        out = self._new("sppf", 4 * x.count, h, w)
        self.step(Step("sppf", (x,), out, (k,)))
        return Ref(out, 0, 4 * x.count)

    # --- modules
    def c2f(self, x_hw: Tuple[int, int], c2: int, n: int, shortcut: bool, x: Optional[Ref] = None) -> Ref:
        h, w = x_hw
        c = c2 // 2
        y = self.conv(2 * c, h, w, src=x)                # cv1
        half = y.count // 2
        parts = [Ref(y.name, y.start, half), Ref(y.name, y.start + half, half)]
        last = parts[-1]
        for _ in range(n):                               # Bottleneck(c, c, shortcut, e=1.0)
            t = self.conv(c, h, w, src=last, k=3)
            t = self.conv(c, h, w, src=t, k=3)
            last = self.add(last, t) if shortcut else t
            parts.append(last)
        cat = self.cat(parts)
        return self.conv(c2, h, w, src=cat)              # cv2

    def sppf(self, hw: Tuple[int, int], c2: int, x: Optional[Ref] = None) -> Ref:
        h, w = hw
        a = self.conv(c2 // 2, h, w, src=x)              # cv1
        pools = self.sppf_pools(a, 5)
        return self.conv(c2, h, w, src=pools)            # cv2


def yolov8s_plan(imgsz: int = 640, nc: int = 80) -> Plan:
    """The non-conv op pass of YOLOv8s at imgsz x imgsz (batch-independent)."""
    if imgsz % 32:
        raise ValueError("imgsz must be a multiple of 32")
    b = _Builder(imgsz, nc)
    s = imgsz
    x = b.conv(32, s // 2, s // 2, k=3, s=2)                     # 0 P1/2
    x = b.conv(64, s // 4, s // 4, src=x, k=3, s=2)              # 1 P2/4
    x = b.c2f((s // 4, s // 4), 64, 1, True, x)                  # 2
    x = b.conv(128, s // 8, s // 8, src=x, k=3, s=2)             # 3 P3/8
    p3 = b.c2f((s // 8, s // 8), 128, 2, True, x)                # 4
    x = b.conv(256, s // 16, s // 16, src=p3, k=3, s=2)          # 5 P4/16
    p4 = b.c2f((s // 16, s // 16), 256, 2, True, x)              # 6
    x = b.conv(512, s // 32, s // 32, src=p4, k=3, s=2)          # 7 P5/32
    x = b.c2f((s // 32, s // 32), 512, 1, True, x)               # 8
    p5 = b.sppf((s // 32, s // 32), 512, x)                      # 9
    up = b.upsample(p5)                                          # 10
    cat = b.cat([up, p4])                                        # 11
    h12 = b.c2f((s // 16, s // 16), 256, 1, False, cat)          # 12
    up = b.upsample(h12)                                         # 13
    cat = b.cat([up, p3])                                        # 14
    o3 = b.c2f((s // 8, s // 8), 128, 1, False, cat)             # 15 (P3 out)
    d = b.conv(128, s // 16, s // 16, src=o3, k=3, s=2)          # 16
    cat = b.cat([d, h12])                                        # 17
    o4 = b.c2f((s // 16, s // 16), 256, 1, False, cat)           # 18 (P4 out)
    d = b.conv(256, s // 32, s // 32, src=o4, k=3, s=2)          # 19
    cat = b.cat([d, p5])                                         # 20
    o5 = b.c2f((s // 32, s // 32), 512, 1, False, cat)           # 21 (P5 out)
    # 22 Detect(nc, ch=(128, 256, 512)): c2 = max(16, 128//4, 64) = 64, c3 = max(128, min(nc, 100))
    c3 = max(128, min(nc, 100))
    anchor = 0
    for stride, feat in ((8, o3), (16, o4), (32, o5)):
        h = w = s // stride
        t = b.conv(64, h, w, src=feat, k=3)
        t = b.conv(64, h, w, src=t, k=3)
        box = b.conv(64, h, w, act=False, src=t)
        t = b.conv(c3, h, w, src=feat, k=3)
        t = b.conv(c3, h, w, src=t, k=3)
        cls = b.conv(nc, h, w, act=False, src=t)
        b.step(Step("restore", (box,), None, (0, 64, anchor)))
        b.step(Step("restore", (cls,), None, (64, nc, anchor)))
        b.plan.levels.append((h, w))
        b.plan.strides.append(float(stride))
        anchor += h * w
    b.step(Step("decode", (), None, (True,)))
    return b.plan


@dataclass(frozen=True)
class ConvSpec:
    """One convolution of the model: input channels, output channels, kernel, stride,
    input height/width, and whether the SiLU epilogue follows (Ultralytics Conv)."""
    cin: int
    cout: int
    k: int
    s: int
    h: int
    w: int
    act: bool = True

    @property
    def out_hw(self) -> Tuple[int, int]:
        p = (self.k - 1) // 2
        return (self.h + 2 * p - self.k) // self.s + 1, (self.w + 2 * p - self.k) // self.s + 1

    @property
    def flops(self) -> int:
        oh, ow = self.out_hw
        return 2 * self.cin * self.cout * self.k * self.k * oh * ow

    @property
    def launches(self) -> int:
        return conv_launches(self.cin, self.cout, self.k, self.s)


def conv_launches(cin: int, cout: int, k: int, stride: int) -> int:
    """Kernels one ``ops.conv2d`` call launches (NC1HWC0 output, no residual): two for
    a stem-shaped conv (one 16-channel input block, 3x3 stride 2, at most 64 outputs:
    the tensor-core and CUDA-core stem kernels, one of which returns at once), else one."""
    return 2 if cin <= C0 and k == 3 and stride == 2 and cout <= 64 else 1


def yolov8s_convs(imgsz: int = 640, nc: int = 80) -> List[ConvSpec]:
    """The 63 convolutions of YOLOv8s at imgsz x imgsz in model order (the same
    topology as yolov8s_plan: C2f cv1 1x1 -> n bottlenecks of two 3x3 -> cv2 1x1 over
    the (2+n) chunks; SPPF 1x1 -> 1x1 over 4 chunks; Detect cv2/cv3 towers of two 3x3 and
    a 1x1 without activation).  The stem's 3 input channels are zero-padded to 16."""
    s = imgsz
    convs: List[ConvSpec] = []

    def conv(cin, cout, k, st, hw, act=True):
        convs.append(ConvSpec(cin, cout, k, st, hw, hw, act))
        return (hw + 2 * ((k - 1) // 2) - k) // st + 1

    def c2f(cin, cout, n, hw):
        c = cout // 2
        conv(cin, 2 * c, 1, 1, hw)
        for _ in range(n):
            conv(c, c, 3, 1, hw)
            conv(c, c, 3, 1, hw)
        conv((2 + n) * c, cout, 1, 1, hw)

    hw = conv(3, 32, 3, 2, s)            # 0
    hw = conv(32, 64, 3, 2, hw)          # 1
    c2f(64, 64, 1, hw)                   # 2
    hw = conv(64, 128, 3, 2, hw)         # 3
    c2f(128, 128, 2, hw)                 # 4
    hw = conv(128, 256, 3, 2, hw)        # 5
    c2f(256, 256, 2, hw)                 # 6
    hw = conv(256, 512, 3, 2, hw)        # 7
    c2f(512, 512, 1, hw)                 # 8
    conv(512, 256, 1, 1, hw)             # 9 SPPF cv1
    conv(1024, 512, 1, 1, hw)            #   SPPF cv2
    c2f(768, 256, 1, s // 16)            # 12
    c2f(384, 128, 1, s // 8)             # 15
    conv(128, 128, 3, 2, s // 8)         # 16
    c2f(384, 256, 1, s // 16)            # 18
    conv(256, 256, 3, 2, s // 16)        # 19
    c2f(768, 512, 1, s // 32)            # 21
    c3 = max(128, min(nc, 100))
    for ch, stride in ((128, 8), (256, 16), (512, 32)):
        hw = s // stride
        conv(ch, 64, 3, 1, hw)
        conv(64, 64, 3, 1, hw)
        conv(64, 64, 1, 1, hw, act=False)
        conv(ch, c3, 3, 1, hw)
        conv(c3, c3, 3, 1, hw)
        conv(c3, nc, 1, 1, hw, act=False)
    return convs


def synthetic_inputs(plan: Plan, batch: int, device, seed: int = 4) -> Dict[str, torch.Tensor]:
    """Seeded N(0,1) fp16 conv outputs, one generator per conv (seed + conv index).

    Drawn in FP32 on ``device`` and rounded to fp16 (on CUDA the stream is the
    Philox generator of that device, on CPU the CPU generator)."""
    device = torch.device(device)
    out = {}
    for index, name in enumerate(plan.conv_inputs):
        c1, h, w = plan.shapes[name]
        g = torch.Generator(device=device)
        g.manual_seed(seed + index)
        out[name] = torch.randn((batch, c1, h, w, C0), generator=g, device=device,
                                dtype=torch.float32).half()
    return out


def concat_placements(plan: Plan):
    """Zero-copy concat plan: for every concat whose inputs are all whole outputs
    of SiLU / residual-add / upsample steps (a C2f ``chunk`` half counts as part of
    its producer), place each producer's output as a C1 slice of the concat
    buffer so it writes there directly, and drop the concat step.

    Returns ({producer: (concat, block offset)}, {elided concat outputs})."""
    producers = {st.output: st for st in plan.steps if st.output is not None}
    placed, elided = {}, set()
    for st in plan.steps:
        if st.op != "cat":
            continue
        local, offset, ok = {}, 0, True
        for ref in st.inputs:
            prod = producers.get(ref.name)
            if prod is None or prod.op not in ("silu", "add", "upsample") or ref.name in placed:
                ok = False
                break
            pos = offset - ref.start
            if local.setdefault(ref.name, pos) != pos:
                ok = False
                break
            offset += ref.count
        if ok:  # placed buffers must tile the concat exactly
            spans = sorted((pos, pos + plan.shapes[name][0]) for name, pos in local.items())
            ok = spans[0][0] == 0 and spans[-1][1] == plan.shapes[st.output][0] and all(
                a[1] == b[0] for a, b in zip(spans, spans[1:]))
        if ok:
            for name, pos in local.items():
                placed[name] = (st.output, pos)
            elided.add(st.output)
    return placed, elided


def silu_add_fusions(plan: Plan) -> Dict[str, Tuple[Ref, Step]]:
    """Residual adds one of whose operands is the whole output of a SiLU step that no
    other step reads: {add output: (the other operand, that SiLU step)}.  In YOLOv8s
    these are the bottlenecks' second conv activations (six adds)."""
    readers: Dict[str, int] = {}
    for st in plan.steps:
        for ref in st.inputs:
            readers[ref.name] = readers.get(ref.name, 0) + 1
    silus = {st.output: st for st in plan.steps if st.op == "silu"}
    out = {}
    for st in plan.steps:
        if st.op != "add":
            continue
        for mine, other in ((st.inputs[1], st.inputs[0]), (st.inputs[0], st.inputs[1])):
            silu = silus.get(mine.name)
            if (silu is not None and readers[mine.name] == 1 and mine.start == 0
                    and mine.count == plan.shapes[mine.name][0]):
                out[st.output] = (other, silu)
                break
    return out


class OpPass:
    """Executes a Plan on one CUDA device with preallocated buffers.

    ``inputs`` maps conv names to [B, c1, h, w, 16] fp16 CUDA tensors (kept
    intact: SiLU writes separate activation buffers, so every run of the pass
    -- and every CUDA-graph replay -- computes the same outputs).
    ``output`` is the decoded [B, 4+nc, anchors] fp16 tensor.

    ``concat_in_place`` turns on the zero-copy concat plan (concat_placements):
    the same tensors result, every concat buffer filled by its producers.
    ``fuse_silu_add`` runs each residual add whose operand is a SiLU output read by
    nothing else as one ``add_silu`` launch on the conv output (silu_add_fusions):
    the add's result is the same, and that SiLU output is never materialised."""

    def __init__(self, plan: Plan, inputs: Dict[str, torch.Tensor], concat_in_place: bool = False,
                 fuse_silu_add: bool = False):
        self.plan = plan
        first = inputs[plan.conv_inputs[0]]
        self.batch = first.size(0)
        self.device = first.device
        self.buffers: Dict[str, torch.Tensor] = dict(inputs)
        self.placed, self.elided = concat_placements(plan) if concat_in_place else ({}, set())
        self.fused = silu_add_fusions(plan) if fuse_silu_add else {}
        skipped = {raw_silu.output for _, raw_silu in self.fused.values()}

        def alloc(name):
            c1, h, w = plan.shapes[name]
            return torch.empty((self.batch, c1, h, w, C0), dtype=torch.float16, device=self.device)

        for name in self.elided:
            self.buffers[name] = alloc(name)
        for name, (cat, pos) in self.placed.items():
            c1 = plan.shapes[name][0]
            self.buffers[name] = self.buffers[cat][:, pos:pos + c1]
        for step in plan.steps:
            if step.output is not None and step.output not in self.buffers and step.output not in skipped:
                self.buffers[step.output] = alloc(step.output)
        self.steps = [st for st in plan.steps
                      if not (st.op == "cat" and st.output in self.elided) and st.output not in skipped]
        self.head = torch.empty((self.batch, 64 + plan.nc, plan.anchors), dtype=torch.float16,
                                device=self.device)
        self.output = torch.empty((self.batch, 4 + plan.nc, plan.anchors), dtype=torch.float16,
                                  device=self.device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def view(self, ref: Ref) -> torch.Tensor:
        t = self.buffers[ref.name]
        if ref.start == 0 and ref.count == t.size(1):
            return t
        return t[:, ref.start:ref.start + ref.count]

    def run_step(self, step: Step) -> None:
        p = self.plan
        if step.op == "silu":
            ops.silu(self.view(step.inputs[0]), out=self.buffers[step.output])
        elif step.op == "add" and step.output in self.fused:
            other, silu = self.fused[step.output]
            ops.add_silu(self.view(other), self.view(silu.inputs[0]), out=self.buffers[step.output])
        elif step.op == "add":
            ops.binary("add", self.view(step.inputs[0]), self.view(step.inputs[1]),
                       out=self.buffers[step.output])
        elif step.op == "cat":
            ops.cat([self.view(r) for r in step.inputs], 1, out=self.buffers[step.output])
        elif step.op == "sppf":
            ops.sppf(self.view(step.inputs[0]), step.attrs[0], out=self.buffers[step.output])
        elif step.op == "upsample":
            ops.upsample_blocked(self.view(step.inputs[0]), out=self.buffers[step.output])
        elif step.op == "restore":
            channel0, channels, anchor0 = step.attrs
            ops.unpack(self.view(step.inputs[0]), channels,
                       out=self.head[:, channel0:channel0 + channels], out_offset=anchor0)
        elif step.op == "decode":
            ops.dfl_decode(self.head[:, :64], self.head[:, 64:], p.levels, p.strides,
                           xywh=step.attrs[0], out=self.output)
        else:
            raise ValueError(step.op)

    def run(self) -> torch.Tensor:
        for step in self.steps:
            self.run_step(step)
        return self.output

    def capture(self, warmup: int = 2) -> torch.cuda.CUDAGraph:
        """Capture the whole pass as one CUDA graph (the FrozenGraph replay path)."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.run()
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.run()
        self.graph = graph
        return graph

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.output

    def launches_per_pass(self) -> int:
        """Kernels one pass launches: one per step, two for the decode (the box
        reduction and the class-row sigmoid, on forked branches)."""
        return sum(2 if step.op == "decode" else 1 for step in self.steps)

    def bytes_per_image(self) -> int:
        """Algorithmic bytes of the steps this pass runs (a fused add moves what the
        add alone does; skipped SiLUs and elided concats move nothing)."""
        return sum(self.plan.step_bytes(step) for step in self.steps)

    def kind(self, step: Step) -> str:
        return "add_silu" if step.op == "add" and step.output in self.fused else step.op


def model_weights(plan: Plan, device, seed: int = 9):
    """Seeded weights for every conv of the plan, one generator per conv (seed + index):
    OIHW fp16 ~ N(0, 2 / fan-in) and bias fp16 ~ N(0, 0.1), drawn in FP32 on the CPU,
    then moved to ``device``."""
    out = []
    for index, name in enumerate(plan.conv_inputs):
        src = plan.conv_sources[index]
        cin = 3 if src is None else src.count * C0
        cout = plan.shapes[name][0] * C0
        k, _ = plan.conv_kernels[index]
        g = torch.Generator().manual_seed(seed + index)
        w = (torch.randn(cout, cin, k, k, generator=g) * (2.0 / (cin * k * k)) ** 0.5).half()
        b = (torch.randn(cout, generator=g) * 0.1).half()
        out.append((w.to(device), b.to(device)))
    return out


def synthetic_image(plan: Plan, batch: int, device, seed: int = 3) -> torch.Tensor:
    """Seeded image batch in NC1HWC0 [B, 1, S, S, 16] fp16: 3 channels ~ U(0, 1), the
    other 13 zero (the stem's input channels padded to one block)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.zeros((batch, 1, plan.imgsz, plan.imgsz, C0), dtype=torch.float16)
    x[..., :3] = torch.rand((batch, 1, plan.imgsz, plan.imgsz, 3), generator=g).half()
    return x.to(device)


class ModelPass(OpPass):
    """The whole YOLOv8s forward on one device: the 63 convolutions (tcgen05 implicit
    GEMM, bias and SiLU fused in the epilogue as the reference's conv does) chained with
    the op pass in model order, capturable as one CUDA graph (the reference's whole-model
    FrozenGraph around its blocked model, blocked_graph.py:4-23, whole_blocked.py:159-327).

    Each activated conv writes its post-SiLU output straight into the op pass's
    activation buffer -- with ``concat_in_place`` that is a C1 slice of the concat it
    feeds -- so the pass's separate SiLU steps are dropped; the Detect box and class
    convs (no activation) write the buffers the restore steps read.  ``weights`` is one
    (OIHW fp16, bias fp16) pair per conv in model order (``model_weights``); ``image``
    is the NC1HWC0 input [B, 1, S, S, 16] (``synthetic_image``).  Class count and every
    conv width must be multiples of 16."""

    def __init__(self, plan: Plan, weights, image: torch.Tensor, concat_in_place: bool = True):
        ops._require(len(weights) == len(plan.conv_inputs), "ModelPass: one (weight, bias) pair per conv")
        ops._require(plan.nc % C0 == 0, "ModelPass: the class count must be a multiple of 16")
        ops._require(image.dtype == torch.float16 and tuple(image.shape[1:]) == (1, plan.imgsz, plan.imgsz, C0),
                     f"ModelPass: image must be fp16 [B, 1, {plan.imgsz}, {plan.imgsz}, 16]")
        self.plan = plan
        self.image = image
        self.batch = image.size(0)
        self.device = image.device
        self.act_of = {st.inputs[0].name: st.output for st in plan.steps if st.op == "silu"}
        self.placed, self.elided = concat_placements(plan) if concat_in_place else ({}, set())
        self.fused = {}  # the convs apply the SiLU themselves

        def alloc(name):
            c1, h, w = plan.shapes[name]
            return torch.empty((self.batch, c1, h, w, C0), dtype=torch.float16, device=self.device)

        self.buffers: Dict[str, torch.Tensor] = {}
        for name in self.elided:
            self.buffers[name] = alloc(name)
        for name, (cat, pos) in self.placed.items():
            self.buffers[name] = self.buffers[cat][:, pos:pos + plan.shapes[name][0]]
        for step in plan.steps:
            if step.output is not None and step.output not in self.buffers:
                self.buffers[step.output] = alloc(step.output)
        self.convs = []
        for index, name in enumerate(plan.conv_inputs):
            out = self.act_of.get(name, name)
            if out not in self.buffers:
                self.buffers[out] = alloc(out)
            w, b = weights[index]
            k, stride = plan.conv_kernels[index]
            self.convs.append((plan.conv_sources[index], ops.conv2d_pack_weights(w.contiguous()), b.contiguous(),
                               int(w.size(0)), k, stride, name in self.act_of, out))
        self.schedule = []
        for kind, index in plan.order:
            if kind == "conv":
                self.schedule.append(("conv", index))
            else:
                step = plan.steps[index]
                if step.op != "silu" and not (step.op == "cat" and step.output in self.elided):
                    self.schedule.append(("step", step))
        self.steps = [item for kind, item in self.schedule if kind == "step"]
        self.head = torch.empty((self.batch, 64 + plan.nc, plan.anchors), dtype=torch.float16,
                                device=self.device)
        self.output = torch.empty((self.batch, 4 + plan.nc, plan.anchors), dtype=torch.float16,
                                  device=self.device)
        self.graph = None

    def conv_input(self, index: int) -> torch.Tensor:
        src = self.convs[index][0]
        return self.image if src is None else self.view(src)

    def run_conv(self, index: int) -> None:
        _, packed, bias, cout, k, stride, silu, out = self.convs[index]
        ops.conv2d(self.conv_input(index), packed, bias, cout, k, stride, silu=silu, out=self.buffers[out])

    def run(self) -> torch.Tensor:
        for kind, item in self.schedule:
            if kind == "conv":
                self.run_conv(item)
            else:
                self.run_step(item)
        return self.output

    def launches_per_pass(self) -> int:
        convs = 0
        for src, _, _, cout, k, stride, _, _ in self.convs:
            convs += conv_launches(3 if src is None else src.count * C0, cout, k, stride)
        return convs + super().launches_per_pass()

    def flops_per_image(self) -> int:
        total = 0
        for index, (src, _, _, cout, k, stride, _, out) in enumerate(self.convs):
            cin = 3 if src is None else src.count * C0
            _, oh, ow = self.plan.shapes[self.plan.conv_inputs[index]]
            total += 2 * cin * cout * k * k * oh * ow
        return total


class C2fRegion:
    """The reference's blocked C2f region (BlockedC2f, blocked_c2f.py:13-24 and
    :83-88; there pinned to YOLOv8s model.6, 256 -> 256 channels at 40x40 with two
    residual bottlenecks) on the tensor cores, with no separate add, cat or unpack pass:

    * cv1 (1x1, c_in -> 2c) writes straight into the concat buffer, whose first two
      c-channel blocks are ``chunk(2, 1)``;
    * bottleneck i runs cv1 (3x3) into a scratch tensor and cv2 (3x3) with the
      residual ``y[-1]`` fused into its epilogue (``y.append(y[-1] + value)``),
      writing its own slice of the concat buffer;
    * cv2 (1x1, (2 + n) c -> c_out) reads the whole buffer and writes NCHW (the
      reference's ``unpack``).

    Every conv is conv + bias + SiLU in FP32 with one fp16 rounding, and the residual
    is fp16(y[-1] + value), so the region equals the reference's op sequence on the
    same weights.  Each conv is given as (OIHW fp16 weight, fp16 bias) on the GPU;
    ``c`` and ``c_out`` must be multiples of 16."""

    def __init__(self, cv1, bottlenecks, cv2, shortcut: bool = True):
        w1, b1 = cv1
        wo, bo = cv2
        _check = ops._require
        _check(w1.dim() == 4 and w1.shape[2:] == (1, 1) and w1.shape[0] % 32 == 0,
               "C2fRegion: cv1 must be 1x1 with 2c outputs, c a multiple of 16")
        self.c_in, self.c = int(w1.shape[1]), int(w1.shape[0]) // 2
        self.n = len(bottlenecks)
        _check(wo.dim() == 4 and wo.shape[2:] == (1, 1) and wo.shape[1] == (2 + self.n) * self.c
               and wo.shape[0] % 16 == 0, "C2fRegion: cv2 must be 1x1 from (2 + n) c channels, c_out % 16 == 0")
        self.c_out = int(wo.shape[0])
        for wa, _, wb, _ in ((a[0], a[1], b[0], b[1]) for a, b in bottlenecks):
            _check(tuple(wa.shape) == (self.c, self.c, 3, 3) and tuple(wb.shape) == (self.c, self.c, 3, 3),
                   "C2fRegion: bottleneck convs must be 3x3 c -> c")
        self.shortcut = shortcut
        self.cv1 = (ops.conv2d_pack_weights(w1), b1)
        self.m = [(ops.conv2d_pack_weights(a[0]), a[1], ops.conv2d_pack_weights(b[0]), b[1])
                  for a, b in bottlenecks]
        self.cv2 = (ops.conv2d_pack_weights(wo), bo)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x: NCHW fp16 [B, c_in, H, W] on the GPU -> NCHW fp16 [B, c_out, H, W]."""
        ops._require(x.dim() == 4 and x.size(1) == self.c_in and x.dtype == torch.float16,
                     f"C2fRegion: expected fp16 NCHW input with {self.c_in} channels")
        b, _, h, w = x.shape
        cb = self.c // C0
        xb = ops.pack(x)
        cat = torch.empty((b, (2 + self.n) * cb, h, w, C0), dtype=torch.float16, device=x.device)
        ops.conv2d(xb, self.cv1[0], self.cv1[1], 2 * self.c, 1, out=cat[:, : 2 * cb])
        scratch = torch.empty((b, cb, h, w, C0), dtype=torch.float16, device=x.device)
        prev = cat[:, cb: 2 * cb]
        for i, (pa, ba, pb, bb) in enumerate(self.m):
            ops.conv2d(prev, pa, ba, self.c, 3, out=scratch)
            dst = cat[:, (2 + i) * cb: (3 + i) * cb]
            ops.conv2d(scratch, pb, bb, self.c, 3, out=dst, residual=prev if self.shortcut else None)
            prev = dst
        return ops.conv2d(cat, self.cv2[0], self.cv2[1], self.c_out, 1, nchw=True, out=out)
