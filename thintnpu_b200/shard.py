"""Image-sharded data parallelism for the op pass (no data-path collective).

Images are independent through the whole op pass, so a batch shards by image:
rank r of G owns the contiguous slice ``shard_range(B, G, r)`` (ceil(B/G)
images, the last rank possibly fewer) and runs the pass on its own GPU.  Nothing
crosses GPUs on the data path; ``torch.distributed`` is only the control plane:
a barrier before/after a timed region and ``max_over_ranks`` for the job time.

Failure detection is host-side: every rank calls ``heartbeat``/``check_peers``
on a TCP store between steps; a rank that raised or stopped is reported to the
others before their next launch (``PeerFailure``), and the process group's short
timeout ends any collective waiting on a dead rank with an error.
"""
from __future__ import annotations

import datetime
import os
import time
from typing import Optional

import torch
import torch.distributed as dist


class PeerFailure(RuntimeError):
    """Another rank reported a failure or stopped sending heartbeats."""


def shard_range(batch: int, world: int, rank: int) -> range:
    """Contiguous image slice of `rank`: ceil(batch/world) images per rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    per = -(-batch // world)
    start = min(batch, rank * per)
    return range(start, min(batch, start + per))


def init(backend: Optional[str] = None, timeout_s: float = 60.0) -> tuple:
    """Join the job described by RANK/WORLD_SIZE/MASTER_ADDR/MASTER_PORT (torchrun)
    with a short timeout; returns (rank, world, local_rank)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return rank, world, local


def max_over_ranks(value: float, device=None) -> float:
    """The job's time: the maximum of a per-rank value (a control-plane all-reduce)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Heartbeat:
    """Host-side liveness between steps on a c10d store (TCP or file).

    ``beat(step)`` records this rank's progress; ``fail(reason)`` publishes a
    failure; ``check(step, wait_s)`` raises PeerFailure if a peer failed or has
    not reached ``step`` within ``wait_s`` seconds."""

    def __init__(self, store, rank: int, world: int):
        self.store, self.rank, self.world = store, rank, world

    def beat(self, step: int) -> None:
        self.store.set(f"hb/{self.rank}", str(step))

    def fail(self, reason: str) -> None:
        self.store.set("hb/failed", f"{self.rank}: {reason}")

    def check_failed(self) -> None:
        """One store round trip: raise PeerFailure if a peer published a failure."""
        if self.store.check(["hb/failed"]):
            raise PeerFailure(self.store.get("hb/failed").decode())

    def step(self, step: int, every: int = 8, wait_s: float = 60.0) -> None:
        """Between steps of a runner: beat `step`, check for a published failure,
        and every `every` steps also wait (up to wait_s) until every rank has
        reached `step`, so no rank runs more than `every` steps ahead of a stopped one."""
        self.beat(step)
        if step % every == 0:
            self.check(step, wait_s)
        else:
            self.check_failed()

    def check(self, step: int, wait_s: float = 5.0) -> None:
        deadline = time.monotonic() + wait_s
        while True:
            if self.store.check(["hb/failed"]):
                raise PeerFailure(self.store.get("hb/failed").decode())
            behind = []
            for r in range(self.world):
                key = f"hb/{r}"
                if not self.store.check([key]) or int(self.store.get(key)) < step:
                    behind.append(r)
            if not behind:
                return
            if time.monotonic() > deadline:
                raise PeerFailure(f"ranks {behind} did not reach step {step} within {wait_s} s")
            time.sleep(0.001)
