"""Workloads and measurement helpers of ``bench.py``.

Each config is one kernel family on its own batch of seeded synthetic data,
inputs resident in HBM (every batch is far above the 126 MB L2, so no flush is
needed between steps), timed with CUDA events on the launching stream over K
steps after W warm-ups, max over ranks.  Configs 1, 2, 3 and 5 capture their K
steps into one CUDA graph and time its replay (the ops run inside a captured pass
in use; eager calls leave ~2.5 µs of host launch gap per kernel in the timing).  The same config objects are what the
GPU parity tests run (tests/test_bench_configs_gpu.py), so the timed
configuration is the tested one.

CPU legs (``cpu_step``) run the oracle -- PyTorch CPU eager, or the numpy
selection restatement -- and are only used for the reported CPU baseline; they
follow one protocol (``cpu_rate``): 3 warm-ups, then the median of at least 11
timed samples.

Multi-GPU: ranks shard images (no data-path collective) and the control plane
(barrier, max over ranks) is a gloo group, so no NCCL communicator exists.
"""
from __future__ import annotations

import json
import os
import statistics
import time
from pathlib import Path

import torch

import thintnpu_b200
from thintnpu_b200 import ops, shard

ROOT = Path(__file__).resolve().parent
METRIC = "non-conv op pass images/s at 640² fp16; achieved HBM GB/s vs ~8 TB/s peak"


def hbm_peak():
    """Measured HBM copy peak of this pool (GB/s) and its kind."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Measured dense bf16 GEMM peak (TFLOP/s, burst) and its kind."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


def gen(shape, seed, device, mean=0.0, std=1.0):
    """Seeded N(mean, std) fp16: drawn in FP32 with the device's own generator
    (Philox on CUDA), then rounded to fp16."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std + mean).half()


def config5_logits(n: int, seed: int = 5, device="cpu", anchors: int = 8400, nc: int = 80) -> torch.Tensor:
    """BASELINE config 5 input: logits [n, 4 + nc, anchors] fp16, channel-planar
    (selection reads the [n, anchors, 4 + nc] transposed view).  Class logits
    ~ N(-4, 2), box rows ~ U(0, 640); per image ~1% of anchors copy another
    anchor's whole class row (exact ties), 0.5% of anchors hold one value across
    all classes, and 8 NaNs (both signs, quiet and signalling payloads) at
    distinct anchors.  The bulk is drawn on `device`; the tie and NaN positions
    come from a seeded CPU generator (distinct targets, so the scatters are
    deterministic)."""
    device = torch.device(device)
    x = gen((n, 4 + nc, anchors), seed, device, mean=-4.0, std=2.0)
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    x[:, :4] = (torch.rand((n, 4, anchors), generator=g, device=device) * 640).half()
    if n == 0 or anchors == 0:
        return x
    c = torch.Generator().manual_seed(seed + 2)
    ties, flat, nans = max(1, anchors // 100), max(1, anchors // 200), min(8, anchors)
    perm = torch.stack([torch.randperm(anchors, generator=c) for _ in range(n)])  # [n, anchors]
    dst = perm[:, :ties]
    src = torch.randint(0, anchors, (n, ties), generator=c)
    rows = perm[:, ties:ties + flat] if ties + flat <= anchors else perm[:, :flat]
    nan_at = perm[:, -nans:]
    nan_cls = torch.randint(0, nc, (n, nans), generator=c)
    b = torch.arange(n, device=device)[:, None]
    dst, src, rows, nan_at, nan_cls = (t.to(device) for t in (dst, src, rows, nan_at, nan_cls))
    view = x.transpose(1, 2)  # [n, anchors, 4 + nc], shares storage with x
    view[b, dst, 4:] = view[b, src, 4:]
    view[b, rows, 4:] = view[b, rows, 4:5]
    payload = torch.tensor([0x7E00, 0xFE00, 0x7C01, 0xFD23, 0x7E01, 0xFFFF, 0x7D00, 0xFC02],
                           dtype=torch.int32).to(torch.int16)[:nans]
    x.view(torch.int16)[b, 4 + nan_cls, nan_at] = payload.to(device).expand(n, nans)
    return x


def cpu_rate(fn, images_per_call: int, warmup: int = 3, samples: int = 11) -> dict:
    """CPU baseline protocol: `warmup` untimed calls, then the median of `samples`
    timed calls (time.perf_counter) under inference_mode; images/s from the median."""
    with torch.inference_mode():
        for _ in range(warmup):
            fn()
        times = []
        for _ in range(samples):
            t = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t)
    med = statistics.median(times)
    return {"value": images_per_call / med, "median_s": med, "samples": samples, "warmup": warmup,
            "total_s": sum(times)}


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or "unknown"."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class Config1:
    """y = SiLU(x + b) + r over NC1HWC0 [B, 8, 80, 80, 16] (bias [128])."""
    name = "config 1: fused SiLU(x+b)+r, NC1HWC0 [B,8,80,80,16] fp16"
    batch, cpu_batch = 256, 4
    bytes_per_image = 3 * 2 * 819200  # x, r read and y written once; the 256-byte bias is per launch
    launches = 1
    graph_steps = True  # timed as one CUDA graph of the K steps, as the op runs inside a captured pass

    def setup(self, batch, device, seed):
        self.x = gen((batch, 8, 80, 80, 16), seed, device)
        self.r = gen((batch, 8, 80, 80, 16), seed + 1, device)
        self.b = gen((128,), seed + 2, device, std=0.1)
        self.y = torch.empty_like(self.x)
        return [self.x, self.r], [self.y]

    def step(self):
        ops.bias_silu_residual(self.x, self.b, self.r, out=self.y)

    def cpu_step(self, batch):
        from oracle import ops as oops
        if not hasattr(self, "cx"):
            g = torch.Generator().manual_seed(1)
            self.cx = torch.randn(batch, 8, 80, 80, 16, generator=g).half()
            self.cr = torch.randn(batch, 8, 80, 80, 16, generator=g).half()
            self.cb = (torch.randn(128, generator=g) * 0.1).half()
        oops.bias_silu_residual(self.cx, self.cb, self.cr)


class Config2:
    """DFL(16) softmax + expectation + anchor decode + sigmoid, [B, 144, 8400] -> [B, 84, 8400]."""
    name = "config 2: Detect decode (DFL softmax, expectation, anchors, sigmoid), A=8400"
    batch, cpu_batch = 256, 2
    shapes, strides = [(80, 80), (40, 40), (20, 20)], [8.0, 16.0, 32.0]
    bytes_per_image = 2 * (64 + 80) * 8400 + 2 * 84 * 8400
    launches = 2
    graph_steps = True  # timed as one CUDA graph of the K steps, as the op runs inside a captured pass

    def setup(self, batch, device, seed):
        self.box = gen((batch, 64, 8400), seed, device, std=2.0)
        self.cls = gen((batch, 80, 8400), seed + 1, device, std=3.0)
        self.out = torch.empty((batch, 84, 8400), dtype=torch.float16, device=device)
        return [self.box, self.cls], [self.out]

    def step(self):
        ops.dfl_decode(self.box, self.cls, self.shapes, self.strides, out=self.out)

    def cpu_step(self, batch):
        from oracle import ops as oops
        if not hasattr(self, "cbox"):
            g = torch.Generator().manual_seed(2)
            self.cbox = (torch.randn(batch, 64, 8400, generator=g) * 2).half()
            self.ccls = (torch.randn(batch, 80, 8400, generator=g) * 3).half()
        oops.dfl_decode(self.cbox, self.ccls, self.shapes, self.strides)


class Config3:
    """C2PSA attention softmax [B, 4, 400, 400], scores scaled by 32^-0.5 (fp16) first."""
    name = "config 3: C2PSA attention row softmax [B,4,400,400] with 32^-0.5 scale"
    batch, cpu_batch = 256, 4
    scale = 32 ** -0.5
    bytes_per_image = 2 * 2 * 4 * 400 * 400
    launches = 1
    graph_steps = True  # timed as one CUDA graph of the K steps, as the op runs inside a captured pass

    def setup(self, batch, device, seed):
        self.x = gen((batch, 4, 400, 400), seed, device)
        self.y = torch.empty_like(self.x)
        return [self.x], [self.y]

    def step(self):
        ops.softmax(self.x, -1, scale=self.scale, out=self.y)

    def cpu_step(self, batch):
        from oracle import ops as oops
        if not hasattr(self, "cx"):
            self.cx = torch.randn(batch, 4, 400, 400, generator=torch.Generator().manual_seed(3)).half()
        oops.softmax(self.cx, -1, scale=self.scale)


class Config5:
    """YOLO26 selection: logits [N, 84, 8400] (transposed view, ties and NaNs as
    the config describes), fp16 sigmoid fused, class max, stable top-k anchors,
    stable top-k pairs (class-aware) or argmax labels (agnostic), packed [N, k, 6]."""
    batch, cpu_batch = 512, 4
    bytes_per_image = 2 * 80 * 8400 + 2 * 4 * 300 + 24 * 300
    launches = 3
    graph_steps = True  # timed as one CUDA graph of the K steps (three launches per call)

    def __init__(self, k: int = 300, agnostic: bool = False, nan_last: bool = False):
        self.k, self.agnostic, self.nan_last = k, agnostic, nan_last
        self.name = (f"config 5: YOLO26 NMS-free selection, [N,8400,84] logits view with ties and NaNs, "
                     f"K={k}, {'agnostic' if agnostic else 'class-aware'}, NaN {'last' if nan_last else 'first'}")
        self.bytes_per_image = 2 * 80 * 8400 + 2 * 4 * k + 24 * k

    def setup(self, batch, device, seed):
        return self.bind(config5_logits(batch, seed, device))

    def bind(self, logits):
        """Select from these logits [N, 84, 8400] (fp16, on the GPU) from now on."""
        batch = logits.size(0)
        self.base = logits
        self.decoded = logits.transpose(1, 2)
        flags = (1 if self.agnostic else 0) | (2 if self.nan_last else 0) | 4
        self.ws = torch.empty(ops.workspace_size(batch, 8400, 80, self.k, flags), dtype=torch.uint8,
                              device=logits.device)
        self.out = torch.empty((batch, self.k, 6), dtype=torch.float32, device=logits.device)
        return [self.base], [self.out]

    def step(self):
        ops.detection_select(self.decoded, self.k, self.agnostic, nan_last=self.nan_last, apply_sigmoid=True,
                             workspace=self.ws, out=self.out)

    def cpu_step(self, batch):
        import numpy as np
        from oracle import select as osel
        if not hasattr(self, "cx"):
            self.cx = config5_logits(batch, 5, "cpu").transpose(1, 2)
        s = self.cx.clone()
        s[..., 4:] = torch.sigmoid(s[..., 4:])
        osel.select(s.contiguous().view(torch.int16).numpy().view(np.uint16), self.k, self.agnostic,
                    self.nan_last)


class Config6:
    """Fused C2PSA attention (beyond the softmax of config 3): q^T k, * 32^-0.5,
    softmax, v attn^T from the qkv conv output [B, 4*(32+32+64), 400]."""
    name = "config 6: fused C2PSA attention, qkv [B,512,400] -> [B,4,64,400], 4 heads, key_dim 32"
    batch, cpu_batch = 512, 8
    heads, kd, hd, n = 4, 32, 64, 400
    scale = 32 ** -0.5
    bytes_per_image = 2 * heads * (2 * kd + hd) * n + 2 * heads * hd * n  # qkv read, out written
    flops_per_image = heads * (2 * n * n * kd + 2 * n * n * hd)
    launches = 1

    def _split(self, qkv):
        return qkv.view(qkv.shape[0], self.heads, 2 * self.kd + self.hd, self.n).split([self.kd, self.kd, self.hd], 2)

    def setup(self, batch, device, seed):
        self.qkv = gen((batch, self.heads * (2 * self.kd + self.hd), self.n), seed, device)
        self.q, self.k, self.v = self._split(self.qkv)
        self.out = torch.empty((batch, self.heads, self.hd, self.n), dtype=torch.float16, device=device)
        return [self.qkv], [self.out]

    def step(self):
        ops.attention(self.q, self.k, self.v, self.scale, out=self.out)

    def cpu_step(self, batch):
        from oracle import ops as oops
        if not hasattr(self, "cqkv"):
            g = torch.Generator().manual_seed(6)
            self.cqkv = torch.randn(batch, self.heads * (2 * self.kd + self.hd), self.n, generator=g).half()
        oops.attention(*self._split(self.cqkv), self.scale)


class Config7:
    """The YOLOv8s-640 conv pass (beyond the op pass): all 63 convolutions with the
    fused bias (+SiLU) epilogue on seeded NC1HWC0 inputs at their true shapes, one
    CUDA-graph replay per step.  Tensor-core bound: 28.6 GFLOP per image."""
    name = "config 7: YOLOv8s-640 conv pass, 63 fused convs (bias+SiLU), NC1HWC0 fp16"
    batch, cpu_batch = 32, 1
    bound = "tensor"

    def __init__(self):
        from thintnpu_b200 import yolo
        self.specs = yolo.yolov8s_convs(640)
        self.launches = sum(sp.launches for sp in self.specs)
        self.flops_per_image = sum(sp.flops for sp in self.specs)
        self.bytes_per_image = sum(2 * 16 * ((sp.cin + 15) // 16) * sp.h * sp.w + 2 * sp.cout * sp.out_hw[0] *
                                   sp.out_hw[1] for sp in self.specs)

    def _layer(self, sp, batch, device, seed):
        g = torch.Generator().manual_seed(seed)
        c1 = (sp.cin + 15) // 16  # NC1HWC0 with the channel tail zero-padded to 16
        x = torch.zeros((batch, c1 * 16, sp.h, sp.w), dtype=torch.float16)
        x[:, : sp.cin] = torch.randn(batch, sp.cin, sp.h, sp.w, generator=g).half()
        x = x.view(batch, c1, 16, sp.h, sp.w).permute(0, 1, 3, 4, 2).contiguous()
        w = (torch.randn(sp.cout, sp.cin, sp.k, sp.k, generator=g) * (sp.cin * sp.k * sp.k) ** -0.5).half()
        b = (torch.randn(sp.cout, generator=g) * 0.1).half()
        return x.to(device), w, b

    def setup(self, batch, device, seed):
        self.layers = []
        for i, sp in enumerate(self.specs):
            x, w, b = self._layer(sp, batch, device, seed + i)
            packed = ops.conv2d_pack_weights(w.to(device))
            oh, ow = sp.out_hw
            out = torch.empty((batch, (sp.cout + 15) // 16, oh, ow, 16), dtype=torch.float16, device=device)
            self.layers.append((sp, x, packed, b.to(device), out))
        self._run()  # first calls size the kernels' shared memory; then capture the pass
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._run()
        return [layer[1] for layer in self.layers], [layer[4] for layer in self.layers]

    def _run(self):
        for sp, x, packed, b, out in self.layers:
            ops.conv2d(x, packed, b, sp.cout, sp.k, sp.s, silu=sp.act, out=out)

    def step(self):
        self.graph.replay()

    def cpu_step(self, batch):
        from oracle import ops as oops
        if not hasattr(self, "clayers"):
            self.clayers = [self._layer(sp, batch, "cpu", 7 + i) for i, sp in enumerate(self.specs)]
        for sp, (x, w, b) in zip(self.specs, self.clayers):
            oops.conv2d(x, w, b, sp.s, sp.act)


class Config8:
    """The depthwise convs of YOLO11s's Detect head at 640 (cv3 towers: DWConv 3x3 + SiLU on
    the level's channels, then on c3 = 128): (128, 80x80) x2, (256 and 128, 40x40),
    (512 and 128, 20x20), NC1HWC0 fp16, one graph replay per step."""
    name = "config 8: YOLO11s-640 Detect depthwise convs, 6 x DWConv 3x3 + SiLU, NC1HWC0 fp16"
    batch, cpu_batch = 64, 2
    shapes = [(128, 80), (128, 80), (256, 40), (128, 40), (512, 20), (128, 20)]
    bytes_per_image = sum(2 * 2 * c * hw * hw for c, hw in shapes)  # read once, written once
    launches = len(shapes)

    def _layer(self, c, hw, batch, seed, device):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(batch, c // 16, hw, hw, 16, generator=g).half()
        w = (torch.randn(c, 1, 3, 3, generator=g) / 3).half()
        b = (torch.randn(c, generator=g) * 0.1).half()
        return x.to(device), w.to(device), b.to(device)

    def setup(self, batch, device, seed):
        self.layers = []
        for i, (c, hw) in enumerate(self.shapes):
            x, w, b = self._layer(c, hw, batch, seed + i, device)
            self.layers.append((x, ops.depthwise_pack_weights(w), b, torch.empty_like(x)))
        self._run()
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._run()
        return [layer[0] for layer in self.layers], [layer[3] for layer in self.layers]

    def _run(self):
        for x, packed, b, out in self.layers:
            ops.depthwise(x, packed, b, 3, 1, silu=True, out=out)

    def step(self):
        self.graph.replay()

    def cpu_step(self, batch):
        from oracle import ops as oops
        if not hasattr(self, "clayers"):
            self.clayers = [self._layer(c, hw, batch, 11 + i, "cpu") for i, (c, hw) in enumerate(self.shapes)]
        for x, w, b in self.clayers:
            oops.depthwise(x, w, b, 3, 1, True)


class Config9:
    """The whole YOLOv8s-640 forward chained on the GPU (yolo.ModelPass): the 63 convs
    with bias + SiLU fused in their epilogue, writing straight into the op pass's
    buffers and concat slices, interleaved with the op pass in model order up to the
    decoded [B, 84, 8400] head, one CUDA-graph replay per step.  Tensor-core bound."""
    name = "config 9: YOLOv8s-640 whole forward, 63 fused convs chained with the op pass, NC1HWC0 fp16"
    batch, cpu_batch = 32, 1
    bound = "tensor"

    def __init__(self):
        from thintnpu_b200 import yolo
        self.plan = yolo.yolov8s_plan(640)
        self.flops_per_image = sum(sp.flops for sp in yolo.yolov8s_convs(640))
        convs = Config7()
        self.bytes_per_image = convs.bytes_per_image + sum(self.plan.bytes_per_image().values())
        self.launches = 0

    def setup(self, batch, device, seed):
        from thintnpu_b200 import yolo
        self.model = yolo.ModelPass(self.plan, yolo.model_weights(self.plan, device, seed),
                                    yolo.synthetic_image(self.plan, batch, device, seed + 1))
        self.launches = self.model.launches_per_pass()
        self.model.capture(warmup=2)
        return [self.model.image], [self.model.output]

    def step(self):
        self.model.graph.replay()

    def cpu_step(self, batch):
        from oracle import yolo as oyolo
        from thintnpu_b200 import yolo
        if not hasattr(self, "cpu_inputs"):
            self.cpu_inputs = (yolo.model_weights(self.plan, "cpu", 9), yolo.synthetic_image(self.plan, batch, "cpu", 10))
        oyolo.run_model(self.plan, *self.cpu_inputs)


CONFIGS = {1: Config1, 2: Config2, 3: Config3, 5: Config5, 6: Config6, 7: Config7, 8: Config8, 9: Config9}


def device_time(step, steps: int, warmup: int, device, barrier, max_over_ranks, graph: bool = False) -> float:
    """Milliseconds of `steps` calls of `step` after `warmup` untimed ones: CUDA
    events on the current stream, a barrier and synchronize on both sides, max
    over ranks.  With `graph` the `steps` calls are captured once into one CUDA
    graph (after the warm-up calls) and the timed region is one replay of it, so
    the host's per-call work stays out of the device time of kernels shorter than
    it; the graph is replayed once untimed first."""
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        step()
    captured = None
    if graph:
        torch.cuda.synchronize(device)
        captured = torch.cuda.CUDAGraph()
        with torch.cuda.graph(captured):
            for _ in range(steps):
                step()
        captured.replay()
        torch.cuda.synchronize(device)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    if captured is not None:
        captured.replay()
    else:
        for _ in range(steps):
            step()
    end.record(stream)
    barrier()
    ms = start.elapsed_time(end)
    del captured
    return max_over_ranks(ms)


def measure_config(cfg, images_total: int, steps: int, warmup: int, device, rank: int, world: int,
                   barrier, max_over_ranks, seed: int) -> dict:
    """One device-timed line for a config with `images_total` images split over the
    ranks (strong scaling: shard_range), roofline against the measured peak."""
    mine = len(shard.shard_range(images_total, world, rank))
    cfg.setup(max(mine, 1), device, seed=seed + rank)
    ms = device_time(cfg.step, steps, warmup, device, barrier, max_over_ranks,
                     graph=getattr(cfg, "graph_steps", False))
    value = images_total * steps / (ms / 1000.0)
    peak, kind = hbm_peak()
    per_gpu_images = -(-images_total // world)
    achieved = cfg.bytes_per_image * per_gpu_images * steps / (ms / 1000.0) / 1e9
    return {"value": value, "unit": "images/s", "images_total": images_total, "images_per_gpu": per_gpu_images,
            "scaling": "strong", "ms_per_step": ms / steps, "steps": steps, "workload": cfg.name,
            "timing": "the K steps as one CUDA graph replay" if getattr(cfg, "graph_steps", False) else "K eager calls",
            "gpu_launches": cfg.launches * steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": f"{kind} hbm_gbs",
                         "how": "algorithmic bytes of the busiest rank's images per step / step time"}}


def unary_sweep(op: str = "silu", sizes_m=(13, 26, 52, 105, 210, 420, 839), reps: int = 10) -> dict:
    """In-place fp16 SiLU/sigmoid bandwidth by tensor size (4 algorithmic bytes per
    element): N(0,1) inputs, 3 warm-ups, then the median of `reps` launches each
    timed with CUDA events after flushing L2 with a 256 MB write."""
    thintnpu_b200.load()
    device = torch.device("cuda", torch.cuda.current_device())
    fn = ops.silu_ if op == "silu" else (lambda t: ops.sigmoid(t, out=t))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    out = {}
    for m in sizes_m:
        x = gen((m * 1000 * 1000,), m, device)
        for _ in range(3):
            fn(x)
        times = []
        for _ in range(reps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn(x)
            e.record()
            torch.cuda.synchronize(device)
            times.append(s.elapsed_time(e))
        t = sorted(times)[len(times) // 2]
        out[f"{m}M"] = {"us": round(t * 1000, 1), "gbs": round(4 * x.numel() / t / 1e6)}
        del x
    return out


def c2f_sweep(batch: int = 32, reps: int = 20) -> dict:
    """YOLOv8s model.6's C2f region (256 -> 256 channels at 40x40, two residual
    bottlenecks; blocked_c2f.py:13-24) fused (``yolo.C2fRegion``) against the same
    op sequence run op by op (pack, conv, chunk, conv, conv, add, cat, conv, unpack),
    seeded random weights; median of ``reps`` CUDA-event timings after 3 warm-ups."""
    from thintnpu_b200.yolo import C2fRegion
    thintnpu_b200.load()
    device = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(1)

    def conv(co, ci, k):
        return ((torch.randn(co, ci, k, k, generator=g) * (1.0 / (ci * k * k) ** 0.5)).half().to(device),
                (torch.randn(co, generator=g) * 0.1).half().to(device))
    cv1, m, cv2 = conv(256, 256, 1), [(conv(128, 128, 3), conv(128, 128, 3)) for _ in range(2)], conv(256, 512, 1)
    region = C2fRegion(cv1, m, cv2)
    x = torch.randn(batch, 256, 40, 40, generator=g).half().to(device)
    packed = {id(w): ops.conv2d_pack_weights(w) for w in [cv1[0], cv2[0]] + [t[0] for pair in m for t in pair]}

    def op_by_op():
        c = lambda t, wb, k, nchw=False: ops.conv2d(t, packed[id(wb[0])], wb[1], wb[0].shape[0], k, nchw=nchw)
        y = list(c(ops.pack(x), cv1, 1).chunk(2, 1))
        for a, b in m:
            prev = y[-1].contiguous()
            y.append(ops.add(prev, c(c(prev, a, 3), b, 3)))
        return ops.unpack(c(ops.cat([t.contiguous() for t in y], 1), cv2, 1))

    out = {"batch": batch}
    for name, fn in (("fused_region", lambda: region(x)), ("op_by_op", op_by_op)):
        for _ in range(3):
            fn()
        times = []
        for _ in range(reps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize(device)
            times.append(s.elapsed_time(e))
        out[name] = round(sorted(times)[len(times) // 2] * 1000, 1)
    return out



def conv_sweep(batch: int = 32, reps: int = 20) -> dict:
    """Each distinct (cin, cout, kernel, stride, input size) of config 7's 63 YOLOv8s
    convolutions at 640 (the stem excepted: it takes ``conv_stem``), timed alone with
    the bias + SiLU epilogue and with the bias only, seeded random NC1HWC0 input and
    weights: ``reps`` calls captured into one CUDA graph after 3 warm-ups, its replay
    between two CUDA events (as the layers run in the model's graph: the host's
    per-call work, ~23 µs, would otherwise set the time of the small layers), with
    the bytes moved once (input + output) and the FLOPs."""
    from thintnpu_b200 import yolo
    thintnpu_b200.load()
    device = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(2)
    shapes = []
    for sp in yolo.yolov8s_convs(640):
        key = (sp.cin, sp.cout, sp.k, sp.s, sp.h)
        if sp.cin >= 16 and key not in shapes:
            shapes.append(key)

    def mean_us(fn):  # over `reps` calls replayed from one graph
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize(device)
        return s.elapsed_time(e) / reps * 1000

    rows = []
    for cin, cout, k, stride, h in shapes:
        x = torch.randn(batch, cin // 16, h, h, 16, generator=g).half().to(device)
        w = (torch.randn(cout, cin, k, k, generator=g) * (2.0 / (cin * k * k)) ** 0.5).half().to(device)
        b = (torch.randn(cout, generator=g) * 0.1).half().to(device)
        packed = ops.conv2d_pack_weights(w)
        out = ops.conv2d(x, packed, b, cout, k, stride)
        oh = out.shape[2]
        silu = mean_us(lambda: ops.conv2d(x, packed, b, cout, k, stride, silu=True, out=out))
        plain = mean_us(lambda: ops.conv2d(x, packed, b, cout, k, stride, silu=False, out=out))
        moved = (x.numel() + out.numel()) * 2
        flops = 2 * batch * oh * oh * cout * cin * k * k
        rows.append({"shape": f"{cin}->{cout} k{k} s{stride} {h}x{h}", "silu_us": round(silu, 1),
                     "bias_only_us": round(plain, 1), "gbs": round(moved / silu / 1e3), "tflops": round(flops / silu / 1e6)})
    torch.cuda.synchronize(device)
    if ops.conv2d_fault():
        raise RuntimeError("conv_sweep: a convolution wait ran out")
    return {"batch": batch, "layers": rows}

def _control_plane(world: int, device):
    """Barrier and max-over-ranks on a gloo group (host tensors; no NCCL)."""
    import torch.distributed as dist

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        return shard.max_over_ranks(v)

    return barrier, max_over_ranks


def run_config(args):
    """``bench.py --config N``: one JSON line for config N on the ranks of this job."""
    cfg = CONFIGS[args.config]()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        threads = getattr(args, "cpu_threads", 0) or os.cpu_count() or 1
        torch.set_num_threads(threads)
        cfg.cpu_step(cfg.cpu_batch)  # builds the inputs
        rate = cpu_rate(lambda: cfg.cpu_step(cfg.cpu_batch), cfg.cpu_batch, warmup=args.warmup,
                        samples=max(args.steps, 11))
        value = rate["value"]
        print(json.dumps({"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
                          "steps": args.steps, "warmup": args.warmup, "impl": "reference",
                          "ms_per_step": 1000 * rate["median_s"], "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                          "config": {"workload": cfg.name, "batch_per_step": cfg.cpu_batch},
                          "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "port",
                                           "sample": f"{cfg.cpu_batch} images per step, PyTorch CPU eager, "
                                                     f"median of {rate['samples']} after {rate['warmup']} warm-ups"},
                          "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    rank, world, local = shard.init("gloo", timeout_s=600)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    thintnpu_b200.load()
    barrier, max_over_ranks = _control_plane(world, device)
    batch = args.batch if args.batch != 256 else cfg.batch
    inputs, outputs = cfg.setup(batch, device, seed=10 * args.config + 1000 * rank)
    graph = bool(getattr(args, "graph_steps", False)) or getattr(cfg, "graph_steps", False)
    ms = device_time(cfg.step, args.steps, args.warmup, device, barrier, max_over_ranks, graph=graph)
    images = world * batch * args.steps
    value = images / (ms / 1000.0)
    tensor = getattr(cfg, "bound", "hbm") == "tensor"
    if tensor:  # TFLOP/s per GPU against the measured dense bf16/fp16 GEMM peak (burst)
        per_gpu = cfg.flops_per_image * batch * args.steps / (ms / 1000.0) / 1e12
        peak, kind = tensor_peak()
    else:
        per_gpu = cfg.bytes_per_image * batch * args.steps / (ms / 1000.0) / 1e9
        peak, kind = hbm_peak()
    # e2e: host copies of the inputs in, results out, every step
    host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in inputs]
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outputs]
    for h, t in zip(host_in, inputs):
        h.copy_(t)

    def e2e_step():
        for h, t in zip(host_in, inputs):
            t.copy_(h, non_blocking=True)
        cfg.step()
        for h, t in zip(host_out, outputs):
            h.copy_(t, non_blocking=True)

    e2e_steps = max(10, args.steps // 4)
    e2e_ms = device_time(e2e_step, e2e_steps, 1, device, barrier, max_over_ranks)
    line = {"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": cfg.name, "batch_per_gpu": batch,
                       "l2": "inputs larger than L2 (no flush needed)",
                       "timing": "the K steps as one CUDA graph replay" if graph else "K eager calls",
                       "algorithmic_bytes_per_image": cfg.bytes_per_image,
                       **({"tensor_flops_per_image": cfg.flops_per_image} if hasattr(cfg, "flops_per_image") else {})},
            "roofline": {"bound": "tensor" if tensor else "hbm", "achieved": per_gpu, "peak": peak,
                         "unit": "TFLOP/s" if tensor else "GB/s", "frac": per_gpu / peak, "peak_kind": kind,
                         "traffic": None},
            "gpu_launches": args.steps * cfg.launches,
            "e2e": {"value": world * batch * e2e_steps / (e2e_ms / 1000.0), "unit": "images/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in inputs),
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in outputs)}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = getattr(args, "cpu_threads", 0) or os.cpu_count() or 1
        torch.set_num_threads(threads)
        cfg.cpu_step(cfg.cpu_batch)
        rate = cpu_rate(lambda: cfg.cpu_step(cfg.cpu_batch), cfg.cpu_batch)
        line["cpu_baseline"] = {"value": rate["value"], "unit": "images/s", "cores": threads, "kind": "port",
                                "sample": f"{cfg.cpu_batch} images per call, PyTorch CPU eager, median of "
                                          f"{rate['samples']} after {rate['warmup']} warm-ups",
                                "cpu_model": cpu_model()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
