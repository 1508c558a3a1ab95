"""Benchmark: YOLOv8s-640 non-conv op pass in images/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ttn|reference]

One process per GPU (torchrun for N > 1).  Each rank owns a fixed shard of
``--batch`` images (weak scaling: images are independent, nothing is exchanged
on the data path); the control plane -- barriers, the max over ranks of the
elapsed time, and host heartbeats between steps -- runs on a gloo group, so no
NCCL communicator is created.  A step is one CUDA-graph replay of the whole op
pass over the rank's batch with every input resident in HBM (inputs are ~14 GB
per step, far above the 126 MB L2, so no flush is needed).  The timed pass is
the zero-copy plan (every concat filled by its producers, bit-identical to the
plain pass, which is reported under ``variants``).

Also reported: ``roofline`` (the SiLU kernel, the pass's dominant kernel),
``sustained`` (the same pass for at least 2 s with its own clock record),
``variants`` (plain pass; config 3 at B=64 and config 5 at N=512, split over the
ranks), ``e2e`` (the pass through the public API with the inputs copied from
pinned host memory and the decoded output read back every step, double
buffered, beside the measured host-to-device copy peak) and, on rank 0 at N=1,
``cpu_baseline`` (the CPU-eager pass, run in a child process with the same
protocol as ``--impl reference``).  ``--impl reference`` times the CPU-eager
pass (the oracle) on the host cores.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
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
WORKLOAD = ("yolov8s-640 non-conv op pass (BASELINE config 4): 57 SiLU, 6 residual adds, 12 C2f/neck concats, "
            "SPPF, 2 upsamples, Detect NCHW restore, DFL decode")
CPU_IMAGES_PER_STEP = 8


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=256, help="images per GPU per step")
    p.add_argument("--imgsz", type=int, default=640)
    p.add_argument("--impl", choices=("ttn", "reference"), default="ttn")
    p.add_argument("--cpu-threads", type=int, default=0,
                   help="host threads of the CPU legs (--impl reference and cpu_baseline; 0 = all)")
    p.add_argument("--cpu-seconds", type=float, default=0.0,
                   help="--impl reference: keep sampling until this much CPU time has been timed")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--sustained-s", type=float, default=2.0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-variants", action="store_true")
    p.add_argument("--graph-steps", action="store_true",
                   help="configs other than 4: time the K steps as one captured CUDA graph (kernels "
                        "shorter than the host's per-call work then run back to back)")
    p.add_argument("--sweep", choices=("silu", "sigmoid", "c2f", "conv"),
                   help="print fp16 unary bandwidth by tensor size, the C2f region fused vs op by op, or "
                        "each config-7 conv shape timed alone (one GPU), and exit")
    p.add_argument("--config", type=int, default=4, choices=(1, 2, 3, 4, 5, 6, 7, 8, 9),
                   help="BASELINE config; 4 (the op pass) is the headline workload; 6 = fused C2PSA attention; "
                        "7 = YOLOv8s conv pass; 8 = YOLO11s depthwise convs; 9 = the whole YOLOv8s forward "
                        "(convs chained with the op pass)")
    return p.parse_args()


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, polled through NVML
    every `period_s` in a thread while a timed region runs (read-only queries)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, torch_index: int, period_s: float = 0.01):
        self.period = period_s
        self.rows = []
        self.handle = None
        self.stop_flag = threading.Event()
        self.thread = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nvml = pynvml
            try:  # the same physical GPU as torch's device index (orders can differ)
                props = torch.cuda.get_device_properties(torch_index)
                bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                visible = os.environ.get("CUDA_VISIBLE_DEVICES")
                index = int(visible.split(",")[torch_index]) if visible else torch_index
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: report the absence
            self.handle = None

    def _poll(self):
        n = self.nvml
        while not self.stop_flag.is_set():
            try:
                self.rows.append((n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM),
                                  n.nvmlDeviceGetCurrentClocksEventReasons(self.handle),
                                  n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0))
            except Exception:
                pass
            self.stop_flag.wait(self.period)

    def start(self):
        if self.handle is not None:
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        return self

    def stop(self) -> dict:
        if self.handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML unavailable"], "samples": 0}
        self.stop_flag.set()
        self.thread.join(timeout=2)
        sm = [r[0] for r in self.rows]
        reasons = sorted({name for r in self.rows for name, bit in self.REASONS.items() if r[1] & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(sm) if sm else None, "reasons": reasons, "samples": len(self.rows),
                "power_w_max": max(r[2] for r in self.rows) if self.rows else None,
                "source": f"NVML every {self.period * 1000:.0f} ms"}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    """--impl reference: the CPU-eager op pass (oracle) on the host cores, rank 0
    only.  A step is CPU_IMAGES_PER_STEP images; W warm-up steps, then at least K
    timed steps (more while --cpu-seconds of timed CPU work is not reached);
    value = images per step / median step time."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch
    from oracle import yolo as oyolo
    from thintnpu_b200 import yolo

    threads = args.cpu_threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    plan = yolo.yolov8s_plan(args.imgsz)
    batch = CPU_IMAGES_PER_STEP
    inputs = yolo.synthetic_inputs(plan, batch, "cpu", seed=4)
    times = []
    with torch.inference_mode():
        for _ in range(args.warmup):
            oyolo.run_pass(plan, inputs)
        while len(times) < args.steps or sum(times) < args.cpu_seconds:
            start = time.perf_counter()
            oyolo.run_pass(plan, inputs)
            times.append(time.perf_counter() - start)
    med = statistics.median(times)
    value = batch / med
    sample = (f"{batch * len(times)} images: {len(times)} steps of {batch} images of the same {args.imgsz} op pass "
              f"(PyTorch CPU eager, with its 12 concat copies), median step after {args.warmup} warm-ups, "
              f"{sum(times):.1f} s timed")
    line = {"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * med, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "batch_per_step": batch, "imgsz": args.imgsz,
                       "sample": f"bounded CPU sample: {batch} images per step"},
            "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "port",
                             "sample": sample, "cpu_model": cpu_model()},
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline(imgsz: int) -> dict:
    """The reference arm's measurement, run in a child process on this host: all
    host threads for at least 10 s of timed CPU work, plus a one-thread sample."""
    def child(threads: int, seconds: float):
        cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "11", "--warmup", "3",
               "--imgsz", str(imgsz), "--cpu-threads", str(threads), "--cpu-seconds", str(seconds)]
        env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
        done = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=600)
        lines = [ln for ln in done.stdout.splitlines() if ln.startswith("{")]
        if done.returncode or not lines:
            raise RuntimeError(f"CPU baseline child failed: {done.stderr[-500:]}")
        return json.loads(lines[-1])["cpu_baseline"]

    every = child(os.cpu_count() or 1, 10.0)
    one = child(1, 3.0)
    every["one_thread"] = {"value": one["value"], "unit": "images/s", "sample": one["sample"]}
    every["protocol"] = "child process of bench.py --impl reference: 3 warm-ups, median of >= 11 steps"
    return every


def main():
    args = parse()
    if args.sweep:
        import bench_configs
        if args.sweep == "c2f":
            print(json.dumps({"sweep": "c2f", "unit": "us", **bench_configs.c2f_sweep()}))
        elif args.sweep == "conv":
            print(json.dumps({"sweep": "conv", "unit": "us", **bench_configs.conv_sweep()}))
        else:
            print(json.dumps({"sweep": args.sweep, "unit": "us / GB/s", **bench_configs.unary_sweep(args.sweep)}))
        return
    if args.config != 4:
        import bench_configs
        bench_configs.run_config(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    run_pass(args)


def run_pass(args):
    import torch
    import torch.distributed as dist

    import bench_configs
    import thintnpu_b200
    from thintnpu_b200 import shard, yolo

    rank, world, local = shard.init("gloo", timeout_s=600)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    thintnpu_b200.load()  # fails loudly without libttn.so
    heartbeat = shard.Heartbeat(dist.distributed_c10d._get_default_store(), rank, world) if world > 1 else None

    plan = yolo.yolov8s_plan(args.imgsz)
    per_image = plan.bytes_per_image()

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def max_over_ranks(value: float) -> float:
        return shard.max_over_ranks(value)

    # --- inputs resident in HBM; rank r owns images shard_range(world*B, world, r)
    images_mine = shard.shard_range(world * args.batch, world, rank)
    inputs = yolo.synthetic_inputs(plan, len(images_mine), device, seed=4 + images_mine.start)
    op_pass = yolo.OpPass(plan, inputs, concat_in_place=True, fuse_silu_add=True)
    op_pass.capture(warmup=2)
    bytes_per_image = op_pass.bytes_per_image()  # no concat copies; no round trip of the fused SiLUs
    stream = torch.cuda.current_stream(device)

    # --- per-op instrumented pass (events on the launching stream) for the roofline
    kinds = {}
    for _ in range(2):
        events = []
        for step in op_pass.steps:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            op_pass.run_step(step)
            e.record(stream)
            events.append((step, s, e))
        torch.cuda.synchronize(device)
    for step, s, e in events:
        k = kinds.setdefault(op_pass.kind(step), {"ms": 0.0, "bytes": 0, "launches": 0})
        k["ms"] += s.elapsed_time(e)
        k["bytes"] += plan.step_bytes(step) * args.batch
        k["launches"] += 1

    # --- timed region: exactly K graph replays, heartbeats between steps
    for _ in range(args.warmup):
        op_pass.replay()
    barrier()
    clocks = ClockSampler(local).start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        op_pass.replay()
        if heartbeat:  # after the step is queued, so the store round trips overlap its work
            heartbeat.step(i)
    end.record(stream)
    barrier()
    clock_info = clocks.stop()
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    images = world * args.batch * args.steps
    value = images / (elapsed_ms / 1000.0)

    # --- sustained: the same replays for >= --sustained-s, with their own clock record
    sustained = None
    if args.sustained_s > 0:
        reps = max(args.steps, math.ceil(args.sustained_s / (elapsed_ms / args.steps / 1000.0)))
        reps = int(max_over_ranks(reps))
        barrier()
        sclocks = ClockSampler(local, period_s=0.05).start()
        ss, se = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ss.record(stream)
        for _ in range(reps):
            op_pass.replay()
        se.record(stream)
        barrier()
        sinfo = sclocks.stop()
        sms = max_over_ranks(ss.elapsed_time(se))
        sustained = {"value": world * args.batch * reps / (sms / 1000.0), "unit": "images/s", "steps": reps,
                     "ms_per_step": sms / reps, "timed_s": sms / 1000.0, "clocks": sinfo}

    # --- variants: the plain pass (concat copies kept); configs 3 and 5 split over the ranks
    variants = {}
    if not args.no_variants:
        plain = yolo.OpPass(plan, inputs)
        plain.capture(warmup=2)
        pms = bench_configs.device_time(plain.replay, args.steps, args.warmup, device, barrier, max_over_ranks)
        pbytes = sum(per_image.values())
        variants["plain_pass"] = {
            "value": images / (pms / 1000.0), "unit": "images/s", "ms_per_step": pms / args.steps,
            "gpu_launches": plain.launches_per_pass() * args.steps, "algorithmic_bytes_per_image": pbytes,
            "achieved_hbm_gbs_pass": pbytes * args.batch * args.steps / (pms / 1000.0) / 1e9,
            "note": "the same pass with the 12 concat copies run as kernels (outputs bit-identical)"}
        plain.graph = None
        del plain
        torch.cuda.empty_cache()
        unfused = yolo.OpPass(plan, inputs, concat_in_place=True)
        unfused.capture(warmup=2)
        ums = bench_configs.device_time(unfused.replay, args.steps, args.warmup, device, barrier, max_over_ranks)
        ubytes = unfused.bytes_per_image()
        variants["zero_copy_unfused"] = {
            "value": images / (ums / 1000.0), "unit": "images/s", "ms_per_step": ums / args.steps,
            "gpu_launches": unfused.launches_per_pass() * args.steps, "algorithmic_bytes_per_image": ubytes,
            "achieved_hbm_gbs_pass": ubytes * args.batch * args.steps / (ums / 1000.0) / 1e9,
            "note": "the zero-copy pass with the six bottleneck SiLUs run as their own kernels "
                    "(outputs bit-identical)"}
        unfused.graph = None
        del unfused
        torch.cuda.empty_cache()
        for key, cfg, total, seed in (("config3_b64", bench_configs.Config3(), 64, 30),
                                      ("config5_n512", bench_configs.Config5(), 512, 50)):
            variants[key] = bench_configs.measure_config(cfg, total, args.steps, args.warmup, device, rank, world,
                                                         barrier, max_over_ranks, seed)
            del cfg
            torch.cuda.empty_cache()

    # --- e2e: public API with host buffers (H2D inputs + D2H output every step)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, plan, op_pass, inputs, device, world, barrier, max_over_ranks)

    peak, peak_kind = bench_configs.hbm_peak()
    silu = kinds["silu"]
    achieved = silu["bytes"] / (silu["ms"] / 1000.0) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch_per_gpu": args.batch, "imgsz": args.imgsz,
                   "parallelism": f"image-sharded x{world}, no data-path collective (gloo control plane)",
                   "l2": "inputs larger than L2 (no flush needed)",
                   "algorithmic_bytes_per_image": bytes_per_image, "replay": "one CUDA graph per step",
                   "concat": "zero-copy: every concat buffer filled in place by its producers (no copy kernels)",
                   "fusion": "the six bottleneck SiLUs run inside their residual adds (ttn_add_silu_f16)"},
        "achieved_hbm_gbs_pass": bytes_per_image * args.batch * args.steps / (elapsed_ms / 1000.0) / 1e9,
        "roofline": {"kernel": f"silu (ttn_silu, {silu['launches']} launches per pass)", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "traffic": silu_traffic_per_launch(plan, op_pass.steps, args.batch),
                     "how": "algorithmic bytes (read+write, 4 B/element) of all SiLU launches of one "
                            "pass / their summed CUDA-event durations"},
        "kernels": {k: {"ms_per_pass": v["ms"], "launches": v["launches"],
                        "gbs": v["bytes"] / (v["ms"] / 1000.0) / 1e9 if v["ms"] else None,
                        "frac": v["bytes"] / (v["ms"] / 1000.0) / 1e9 / peak if v["ms"] else None}
                    for k, v in kinds.items()},
        "gpu_launches": op_pass.launches_per_pass() * args.steps,
        "clocks": clock_info,
        "sustained": sustained,
        "e2e": e2e,
        "variants": variants,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.imgsz)
    if rank == 0:
        print(json.dumps(line), flush=True)
    op_pass.graph = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def silu_traffic_per_launch(plan, steps, batch):
    """DRAM bytes of the average SiLU launch of the pass (`steps`, the ones it runs),
    scaled from the committed ncu capture's bytes per element (profiles/silu_f16.json)."""
    path = ROOT / "profiles" / "silu_f16.json"
    if not path.exists():
        return None
    per_element = float(json.loads(path.read_text())["dram_bytes_per_element"])
    silu_steps = [s for s in steps if s.op == "silu"]
    elements = sum(plan.elements(s.inputs[0].name) for s in silu_steps)
    return per_element * elements * batch / len(silu_steps)


def run_e2e(args, plan, op_pass, inputs, device, world, barrier, max_over_ranks):
    """The pass through the public API with host buffers, double buffered: every
    step copies all of the step's conv outputs host->device from pinned memory
    (copy stream), replays the pass on them (compute stream) and reads the decoded
    output back (a second copy stream).  Step i+1's inputs go into the other of
    two device input sets while step i runs.  The pinned source is one pool per
    rank of at most a quarter of the free host RAM split over the local ranks;
    inputs larger than the pool are copied from it chunk by chunk, so the bytes
    crossing PCIe per step are always the full input set.  Before the timed steps,
    every rank copies 4 GiB from the pool at once (256 MiB copies) to measure the
    concurrent host-to-device copy peak."""
    import psutil
    import torch

    from thintnpu_b200 import yolo
    names = plan.conv_inputs
    step_bytes = sum(inputs[n].numel() * 2 for n in names)
    local_ranks = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    budget = int(0.25 * psutil.virtual_memory().available / local_ranks)
    pool_elems = max(1 << 28, min(step_bytes, budget) // 2)
    pool = torch.empty(pool_elems, dtype=torch.float16, pin_memory=True)
    filled = 0
    for n in names:  # the pool holds real conv outputs
        take = min(inputs[n].numel(), pool_elems - filled)
        pool[filled:filled + take].copy_(inputs[n].reshape(-1)[:take])
        filled += take
        if filled == pool_elems:
            break
    second = {n: torch.empty_like(t) for n, t in inputs.items()}
    passes = [op_pass, yolo.OpPass(plan, second, concat_in_place=True, fuse_silu_add=True)]
    passes[1].capture(warmup=1)
    results = [torch.empty(p.output.shape, dtype=torch.float16, pin_memory=True) for p in passes]
    compute = torch.cuda.current_stream(device)
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)

    # concurrent host->device copy peak (all ranks at once)
    dst = inputs[names[0]].reshape(-1)
    chunk = min(1 << 27, pool_elems, dst.numel())
    total = 0
    barrier()
    ps, pe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ps.record(h2d)
    with torch.cuda.stream(h2d):
        while total < (4 << 30):
            dst[:chunk].copy_(pool[:chunk], non_blocking=True)
            total += 2 * chunk
    pe.record(h2d)
    barrier()
    peak_ms = max_over_ranks(ps.elapsed_time(pe))
    h2d_peak = world * total / (peak_ms / 1000.0) / 1e9

    offset = [0]

    def upload(p):
        """H2D of one step's inputs into pass p's input set, on the copy stream."""
        for n in names:
            t = p.buffers[n].reshape(-1)
            done = 0
            while done < t.numel():
                take = min(t.numel() - done, pool_elems - offset[0])
                t[done:done + take].copy_(pool[offset[0]:offset[0] + take], non_blocking=True)
                done += take
                offset[0] = (offset[0] + take) % pool_elems

    def run(steps: int) -> float:
        uploaded = [torch.cuda.Event() for _ in passes]
        replayed = [torch.cuda.Event() for _ in passes]
        read = [torch.cuda.Event() for _ in passes]
        for e in replayed + read:
            e.record(compute)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(compute)
        h2d.wait_event(start)
        for i in range(steps + 1):
            if i < steps:  # inputs of step i: wait until step i-2 has finished reading this set
                j = i % 2
                h2d.wait_event(replayed[j])
                with torch.cuda.stream(h2d):
                    upload(passes[j])
                uploaded[j].record(h2d)
            if i > 0:  # replay step i-1 (its inputs landed, its output buffer was read back)
                j = (i - 1) % 2
                compute.wait_event(uploaded[j])
                compute.wait_event(read[j])
                passes[j].replay()
                replayed[j].record(compute)
                d2h.wait_event(replayed[j])
                with torch.cuda.stream(d2h):
                    results[j].copy_(passes[j].output, non_blocking=True)
                read[j].record(d2h)
        for e in read:
            compute.wait_event(e)
        end.record(compute)
        return start, end

    run(1)
    barrier()
    start, end = run(args.e2e_steps)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    value = world * args.batch * args.e2e_steps / (ms / 1000.0)
    out = {"value": value, "unit": "images/s", "h2d_bytes_per_step": step_bytes,
           "d2h_bytes_per_step": results[0].numel() * 2, "steps": args.e2e_steps,
           "h2d_gbs": world * step_bytes * args.e2e_steps / (ms / 1000.0) / 1e9,
           "h2d_peak_gbs": h2d_peak,
           "pinned_pool_bytes": pool_elems * 2,
           "path": "pinned host pool -> cudaMemcpyAsync per conv output (copy stream) -> graph replay "
                   "(compute stream, two input sets) -> pinned host (second copy stream)"}
    out["h2d_frac_of_peak"] = out["h2d_gbs"] / h2d_peak
    for p in passes[1:]:
        p.graph = None
    return out


if __name__ == "__main__":
    main()
