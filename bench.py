"""Benchmark: YOLOv8s-640 non-conv op pass in images/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ttn|reference]

One process per GPU (torchrun for N > 1).  Each rank owns a fixed shard of
``--batch`` images (weak scaling: images are independent, nothing is
exchanged on the data path; a tiny all-reduce only takes the max time).  A
step is one CUDA-graph replay of the whole op pass over the rank's batch with
all inputs resident in HBM (inputs are ~14 GB per step, far above the 126 MB
L2, so no flush is needed).  ``e2e`` times the same pass through the public
API with the inputs copied from pinned host memory and the decoded output read
back every step.  ``--impl reference`` times the CPU-eager pass (the oracle)
on the host cores instead.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "non-conv op pass images/s at 640² fp16; achieved HBM GB/s vs ~8 TB/s peak"
WORKLOAD = "yolov8s-640 non-conv op pass (BASELINE config 4): 57 SiLU, 6 residual adds, 12 C2f/neck concats, SPPF, 2 upsamples, Detect NCHW restore, DFL decode"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=256, help="images per GPU per step")
    p.add_argument("--imgsz", type=int, default=640)
    p.add_argument("--impl", choices=("ttn", "reference"), default="ttn")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-variants", action="store_true")
    p.add_argument("--sweep", choices=("silu", "sigmoid", "c2f"),
                   help="print fp16 unary bandwidth by tensor size, or the C2f region fused vs op by op "
                        "(one GPU), and exit")
    p.add_argument("--config", type=int, default=4, choices=(1, 2, 3, 4, 5, 6, 7, 8),
                   help="BASELINE config; 4 (the op pass) is the headline workload; 6 = fused C2PSA attention; 7 = YOLOv8s conv pass; 8 = YOLO11s depthwise convs")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or "unknown"."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_pass_rate(imgsz: int, budget_s: float = 12.0, one_thread_s: float = 5.0):
    """CPU-eager op pass (the oracle) on the host cores: images/s over a bounded
    sample with every core, plus a shorter sample on one thread."""
    import torch
    from oracle import yolo as oyolo
    from thintnpu_b200 import yolo

    plan = yolo.yolov8s_plan(imgsz)
    batch = 2
    inputs = yolo.synthetic_inputs(plan, batch, "cpu", seed=4)

    def rate(threads: int, budget: float):
        torch.set_num_threads(threads)
        with torch.inference_mode():
            oyolo.run_pass(plan, inputs)  # warm-up
            done, start = 0, time.perf_counter()
            while True:
                oyolo.run_pass(plan, inputs)
                done += batch
                elapsed = time.perf_counter() - start
                if elapsed >= budget:
                    return done, elapsed

    cores = os.cpu_count() or 1
    done, elapsed = rate(cores, budget_s)
    done1, elapsed1 = rate(1, one_thread_s)
    torch.set_num_threads(cores)
    return {"value": done / elapsed, "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"{done} images ({batch} per pass) of the same {imgsz} op pass, PyTorch CPU eager, "
                      f"{elapsed:.1f} s",
            "one_thread": {"value": done1 / elapsed1, "unit": "images/s",
                           "sample": f"{done1} images, {elapsed1:.1f} s"},
            "cpu_model": cpu_model()}


def run_reference(args):
    """--impl reference: the CPU-eager pass on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from oracle import yolo as oyolo
    from thintnpu_b200 import yolo

    torch.set_num_threads(os.cpu_count() or 1)
    plan = yolo.yolov8s_plan(args.imgsz)
    batch = 2
    inputs = yolo.synthetic_inputs(plan, batch, "cpu", seed=4)
    times = []
    with torch.inference_mode():
        for i in range(args.warmup + args.steps):
            start = time.perf_counter()
            oyolo.run_pass(plan, inputs)
            if i >= args.warmup:
                times.append(time.perf_counter() - start)
    total = sum(times)
    value = batch * len(times) / total
    line = {"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * total / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "batch_per_step": batch, "imgsz": args.imgsz,
                       "sample": "bounded CPU sample: 2 images per step"},
            "cpu_baseline": {"value": value, "unit": "images/s", "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": f"{batch * len(times)} images, PyTorch CPU eager op pass (oracle)"},
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.sweep:
        from thintnpu_b200 import perf
        if args.sweep == "c2f":
            print(json.dumps({"sweep": "c2f", "unit": "us", **perf.c2f_sweep()}))
        else:
            print(json.dumps({"sweep": args.sweep, "unit": "us / GB/s", **perf.unary_sweep(args.sweep)}))
        return
    if args.config != 4:
        from thintnpu_b200 import perf
        perf.run_config(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from thintnpu_b200 import shard
    rank, world, local = shard.init("nccl", timeout_s=600)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)

    import thintnpu_b200
    thintnpu_b200.load()  # fails loudly without libttn.so
    from thintnpu_b200 import yolo

    plan = yolo.yolov8s_plan(args.imgsz)
    per_image = plan.bytes_per_image()
    bytes_per_image = sum(per_image.values())

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def max_over_ranks(value: float) -> float:
        return shard.max_over_ranks(value, device)

    # --- inputs resident in HBM; rank r owns images shard_range(world*B, world, r)
    images_mine = shard.shard_range(world * args.batch, world, rank)
    inputs = yolo.synthetic_inputs(plan, len(images_mine), device, seed=4 + images_mine.start)
    op_pass = yolo.OpPass(plan, inputs)
    op_pass.capture(warmup=2)
    stream = torch.cuda.current_stream(device)

    # --- per-op instrumented pass (events on the launching stream) for the roofline
    kinds = {}
    for _ in range(2):
        events = []
        for step in plan.steps:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            op_pass.run_step(step)
            e.record(stream)
            events.append((step, s, e))
        torch.cuda.synchronize(device)
    for step, s, e in events:
        k = kinds.setdefault(step.op, {"ms": 0.0, "bytes": 0, "launches": 0})
        k["ms"] += s.elapsed_time(e)
        k["bytes"] += plan.step_bytes(step) * args.batch
        k["launches"] += 1

    # --- timed region: K graph replays
    for _ in range(args.warmup):
        op_pass.replay()
    barrier()
    clocks = ClockSampler(local) if local == 0 or world == 1 else None
    if clocks:
        clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        op_pass.replay()
    end.record(stream)
    barrier()
    clock_info = clocks.stop() if clocks else None
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    images = world * args.batch * args.steps
    value = images / (elapsed_ms / 1000.0)

    # --- variant: zero-copy concat plan (producers write into concat slices)
    variants = {}
    if not args.no_variants:
        zc = yolo.OpPass(plan, inputs, concat_in_place=True)
        zc.capture(warmup=2)
        for _ in range(args.warmup):
            zc.replay()
        barrier()
        zs, ze = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        zs.record(stream)
        for _ in range(args.steps):
            zc.replay()
        ze.record(stream)
        barrier()
        zms = max_over_ranks(zs.elapsed_time(ze))
        zbytes = bytes_per_image - per_image.get("cat", 0)
        variants["concat_in_place"] = {
            "value": images / (zms / 1000.0), "unit": "images/s", "ms_per_step": zms / args.steps,
            "gpu_launches": zc.launches_per_pass() * args.steps,
            "algorithmic_bytes_per_image": zbytes,
            "achieved_hbm_gbs_pass": zbytes * images / world / (zms / 1000.0) / 1e9,
            "note": "same outputs bit for bit; the 12 concat copies are elided by placing each "
                    "producer's output in its concat slice"}
        zc.graph = None
        del zc

    # --- e2e: public API with host buffers (H2D inputs + D2H output every step)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, plan, op_pass, device, stream, world, barrier, max_over_ranks)

    peak, peak_kind = peaks()
    silu = kinds["silu"]
    achieved = silu["bytes"] / (silu["ms"] / 1000.0) / 1e9
    traffic = silu_traffic_per_launch(plan, args.batch)
    line = {
        "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch_per_gpu": args.batch, "imgsz": args.imgsz,
                   "parallelism": f"image-sharded x{world}, no data-path collective",
                   "l2": "inputs larger than L2 (no flush needed)",
                   "algorithmic_bytes_per_image": bytes_per_image, "replay": "one CUDA graph per step"},
        "achieved_hbm_gbs_pass": bytes_per_image * value / world / 1e9,
        "roofline": {"kernel": "silu (ttn_silu, 57 launches per pass)", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "traffic": traffic,
                     "how": "algorithmic bytes (read+write, 4 B/element) of all SiLU launches of one "
                            "pass / their summed CUDA-event durations"},
        "kernels": {k: {"ms_per_pass": v["ms"], "launches": v["launches"],
                        "gbs": v["bytes"] / (v["ms"] / 1000.0) / 1e9 if v["ms"] else None}
                    for k, v in kinds.items()},
        "gpu_launches": op_pass.launches_per_pass() * args.steps,
        "clocks": clock_info,
        "e2e": e2e,
        "variants": variants,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_pass_rate(args.imgsz)
    if rank == 0:
        print(json.dumps(line), flush=True)
    op_pass.graph = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def silu_traffic_per_launch(plan, batch):
    """DRAM bytes of the average SiLU launch, scaled from the committed ncu capture
    (profiles/silu_f16.md: `dram_bytes_per_element: X`), else None."""
    path = ROOT / "profiles" / "silu_f16.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_element:"):
            per_element = float(line.split(":", 1)[1])
            elements = sum(plan.elements(s.inputs[0].name) for s in plan.steps if s.op == "silu")
            launches = sum(1 for s in plan.steps if s.op == "silu")
            return per_element * elements * batch / launches
    return None


def run_e2e(args, plan, op_pass, device, stream, world, barrier, max_over_ranks):
    """Same pass through the public API with host buffers: every step copies all of
    the step's conv outputs host->device from pinned memory, replays the pass and
    reads the decoded output back.  The pinned source is one pool per rank of at
    most a quarter of the free host RAM split over the local ranks; inputs larger
    than the pool are copied from it chunk by chunk, so the bytes crossing PCIe
    per step are always the full input set."""
    import psutil
    import torch
    names = plan.conv_inputs
    step_bytes = sum(op_pass.buffers[n].numel() * 2 for n in names)
    local_ranks = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    budget = int(0.25 * psutil.virtual_memory().available / local_ranks)
    pool_elems = max(1 << 20, min(step_bytes, budget) // 2)
    pool = torch.empty(pool_elems, dtype=torch.float16, pin_memory=True)
    pool.copy_(op_pass.buffers[names[0]].reshape(-1)[:pool_elems]
               if op_pass.buffers[names[0]].numel() >= pool_elems else
               torch.randn(pool_elems, dtype=torch.float32).half())
    result = torch.empty(op_pass.output.shape, dtype=torch.float16, pin_memory=True)

    def step():
        offset = 0
        for n in names:  # H2D of this step's inputs
            dst = op_pass.buffers[n].reshape(-1)
            done = 0
            while done < dst.numel():
                take = min(dst.numel() - done, pool_elems - offset)
                dst[done:done + take].copy_(pool[offset:offset + take], non_blocking=True)
                done += take
                offset = (offset + take) % pool_elems
        op_pass.replay()
        result.copy_(op_pass.output, non_blocking=True)  # D2H of the step's result

    step()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.e2e_steps):
        step()
    end.record(stream)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    value = world * args.batch * args.e2e_steps / (ms / 1000.0)
    return {"value": value, "unit": "images/s", "h2d_bytes_per_step": step_bytes,
            "d2h_bytes_per_step": result.numel() * 2, "steps": args.e2e_steps,
            "pinned_pool_bytes": pool_elems * 2,
            "path": "pinned host pool -> cudaMemcpyAsync per conv output -> graph replay -> pinned host"}


if __name__ == "__main__":
    main()
