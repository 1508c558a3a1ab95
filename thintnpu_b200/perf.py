"""Per-config measurements for BASELINE configs 1, 2, 3 and 5, and 6 = the fused
C2PSA attention built on config 3's softmax (``bench.py --config N``).

Each config is one kernel family on its own batch, inputs resident in HBM
(every batch is far above the 126 MB L2), timed with CUDA events on the
launching stream over K steps after W warm-ups, max over ranks.  The printed
JSON line has the bench.py keys: value (images/s over all GPUs), roofline
(algorithmic bytes per step / step time vs the measured HBM copy peak), e2e
(host buffers copied in and results read back every step) and, on rank 0 at
N=1, the CPU-eager baseline on a bounded sample.
"""
from __future__ import annotations

import json
import os
import time
from pathlib import Path

import torch

from . import ops

ROOT = Path(__file__).resolve().parent.parent
METRIC = "non-conv op pass images/s at 640² fp16; achieved HBM GB/s vs ~8 TB/s peak"


def _peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _tensor_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


def _gen(shape, seed, device, mean=0.0, std=1.0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std + mean).half()


class Config1:
    """y = SiLU(x + b) + r over NC1HWC0 [B, 8, 80, 80, 16] (bias [128])."""
    name = "config 1: fused SiLU(x+b)+r, NC1HWC0 [B,8,80,80,16] fp16"
    batch, cpu_batch = 256, 4
    bytes_per_image = 3 * 2 * 819200  # x, r read and y written once; the 256-byte bias is per launch

    def setup(self, batch, device, seed):
        self.x = _gen((batch, 8, 80, 80, 16), seed, device)
        self.r = _gen((batch, 8, 80, 80, 16), seed + 1, device)
        self.b = _gen((128,), seed + 2, device, std=0.1)
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

    def setup(self, batch, device, seed):
        self.box = _gen((batch, 64, 8400), seed, device, std=2.0)
        self.cls = _gen((batch, 80, 8400), seed + 1, device, std=3.0)
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

    def setup(self, batch, device, seed):
        self.x = _gen((batch, 4, 400, 400), seed, device)
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
    """YOLO26 selection: logits [N, 84, 8400] (transposed view), fp16 sigmoid fused,
    class max, stable top-300 anchors, stable top-300 pairs, packed [N, 300, 6]."""
    name = "config 5: YOLO26 NMS-free selection, [N,8400,84] logits view, K=300, class-aware"
    batch, cpu_batch = 512, 4
    k = 300
    bytes_per_image = 2 * 80 * 8400 + 2 * 4 * 300 + 24 * 300

    def setup(self, batch, device, seed):
        x = _gen((batch, 84, 8400), seed, device, mean=-4.0, std=2.0)
        x[:, :4] = (torch.rand((batch, 4, 8400), device=device) * 640).half()
        self.base = x
        self.decoded = x.transpose(1, 2)
        self.ws = torch.empty(ops.workspace_size(batch, 8400, 80, self.k, 4), dtype=torch.uint8, device=device)
        self.out = torch.empty((batch, self.k, 6), dtype=torch.float32, device=device)
        return [self.base], [self.out]

    def step(self):
        ops.detection_select(self.decoded, self.k, False, apply_sigmoid=True, workspace=self.ws,
                             out=self.out)

    def cpu_step(self, batch):
        import numpy as np
        from oracle import select as osel
        if not hasattr(self, "cbits"):
            g = torch.Generator().manual_seed(5)
            x = (torch.randn(batch, 84, 8400, generator=g) * 2 - 4).half()
            self.cx = x.transpose(1, 2)
        s = self.cx.clone()
        s[..., 4:] = torch.sigmoid(s[..., 4:])
        osel.select(s.contiguous().view(torch.int16).numpy().view(np.uint16), self.k)


class Config6:
    """Fused C2PSA attention (beyond the softmax of config 3): q^T k, * 32^-0.5,
    softmax, v attn^T from the qkv conv output [B, 4*(32+32+64), 400]."""
    name = "config 6: fused C2PSA attention, qkv [B,512,400] -> [B,4,64,400], 4 heads, key_dim 32"
    batch, cpu_batch = 512, 8
    heads, kd, hd, n = 4, 32, 64, 400
    scale = 32 ** -0.5
    bytes_per_image = 2 * heads * (2 * kd + hd) * n + 2 * heads * hd * n  # qkv read, out written
    flops_per_image = heads * (2 * n * n * kd + 2 * n * n * hd)

    def _split(self, qkv):
        return qkv.view(qkv.shape[0], self.heads, 2 * self.kd + self.hd, self.n).split([self.kd, self.kd, self.hd], 2)

    def setup(self, batch, device, seed):
        self.qkv = _gen((batch, self.heads * (2 * self.kd + self.hd), self.n), seed, device)
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
        from . import yolo
        self.specs = yolo.yolov8s_convs(640)
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
    specs = shapes

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


CONFIGS = {1: Config1, 2: Config2, 3: Config3, 5: Config5, 6: Config6, 7: Config7, 8: Config8}


def unary_sweep(op: str = "silu", sizes_m=(13, 26, 52, 105, 210, 420, 839), reps: int = 10) -> dict:
    """In-place fp16 SiLU/sigmoid bandwidth by tensor size (4 algorithmic bytes per
    element): N(0,1) inputs, 3 warm-ups, then the median of `reps` launches each
    timed with CUDA events after flushing L2 with a 256 MB write."""
    import thintnpu_b200
    thintnpu_b200.load()
    device = torch.device("cuda", torch.cuda.current_device())
    fn = ops.silu_ if op == "silu" else (lambda t: ops.sigmoid(t, out=t))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    out = {}
    for m in sizes_m:
        x = _gen((m * 1000 * 1000,), m, device)
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
    import thintnpu_b200
    from .yolo import C2fRegion
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


def run_config(args):
    import torch.distributed as dist
    cfg = CONFIGS[args.config]()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        torch.set_num_threads(os.cpu_count() or 1)
        with torch.inference_mode():
            cfg.cpu_step(cfg.cpu_batch)
            times = []
            for _ in range(args.steps):
                t = time.perf_counter()
                cfg.cpu_step(cfg.cpu_batch)
                times.append(time.perf_counter() - t)
        value = cfg.cpu_batch * len(times) / sum(times)
        print(json.dumps({"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
                          "steps": args.steps, "warmup": args.warmup, "impl": "reference",
                          "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                          "config": {"workload": cfg.name, "batch_per_step": cfg.cpu_batch},
                          "cpu_baseline": {"value": value, "unit": "images/s",
                                           "cores": torch.get_num_threads(), "kind": "port",
                                           "sample": f"{cfg.cpu_batch} images per step, PyTorch CPU eager"},
                          "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    import thintnpu_b200
    thintnpu_b200.load()
    batch = args.batch if args.batch != 256 else cfg.batch
    inputs, outputs = cfg.setup(batch, device, seed=10 * args.config + 1000 * rank)
    stream = torch.cuda.current_stream(device)

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        cfg.step()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        cfg.step()
    end.record(stream)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    images = world * batch * args.steps
    value = images / (ms / 1000.0)
    peak, kind = _peak()
    achieved = cfg.bytes_per_image * batch * args.steps / (ms / 1000.0) / 1e9 / 1.0
    per_gpu = achieved / world
    tensor = getattr(cfg, "bound", "hbm") == "tensor"
    if tensor:  # TFLOP/s per GPU against the measured dense bf16/fp16 GEMM peak (burst)
        per_gpu = cfg.flops_per_image * batch * args.steps / (ms / 1000.0) / 1e12 / world
        peak, kind = _tensor_peak()
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

    e2e_step()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    for _ in range(max(2, args.steps // 4)):
        e2e_step()
    e2.record(stream)
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))
    e2e_steps = max(2, args.steps // 4)
    line = {"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": cfg.name, "batch_per_gpu": batch,
                       "l2": "inputs larger than L2 (no flush needed)",
                       "algorithmic_bytes_per_image": cfg.bytes_per_image,
                       **({"tensor_flops_per_image": cfg.flops_per_image} if hasattr(cfg, "flops_per_image") else {})},
            "roofline": {"bound": "tensor" if tensor else "hbm", "achieved": per_gpu, "peak": peak,
                         "unit": "TFLOP/s" if tensor else "GB/s", "frac": per_gpu / peak, "peak_kind": kind,
                         "traffic": None},
            "gpu_launches": args.steps * (4 if args.config == 5 else len(getattr(cfg, "specs", [0]))),
            "e2e": {"value": world * batch * e2e_steps / (e2e_ms / 1000.0), "unit": "images/s",
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in inputs),
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in outputs)}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        with torch.inference_mode():
            cfg.cpu_step(cfg.cpu_batch)
            done, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < 10.0:
                cfg.cpu_step(cfg.cpu_batch)
                done += cfg.cpu_batch
            el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": done / el, "unit": "images/s", "cores": torch.get_num_threads(),
                                "kind": "port", "sample": f"{done} images, PyTorch CPU eager, {el:.1f} s"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
