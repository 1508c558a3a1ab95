"""CPU (gloo, world size 2): image sharding, max-over-ranks timing, and host-side
failure detection of the multi-GPU runner -- no GPU, nothing faulted."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp

from thintnpu_b200.shard import shard_range


def test_shard_ranges_cover_every_image_once():
    for batch in (0, 1, 7, 256, 257, 512):
        for world in (1, 2, 4, 8):
            seen = []
            for rank in range(world):
                r = shard_range(batch, world, rank)
                assert len(r) <= -(-batch // world) if batch else len(r) == 0
                seen.extend(r)
            assert seen == list(range(batch))
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from thintnpu_b200 import shard
    rank_, world_, _ = shard.init("gloo", timeout_s=20)
    store = dist.distributed_c10d._get_default_store()
    hb = shard.Heartbeat(store, rank_, world_)
    try:
        if mode == "max":
            results[rank] = shard.max_over_ranks(10.0 + rank)
        elif mode == "raise":
            hb.beat(0)
            if rank == 1:
                hb.check(0)
                hb.fail("injected exception in step 1")
                raise RuntimeError("injected")
            try:  # rank 0 may still be in its step-0 check when the failure lands
                hb.check(0, wait_s=10)
                hb.check(1, wait_s=10)
                results[rank] = "missed"
            except shard.PeerFailure as err:
                results[rank] = f"detected: {err}"
        elif mode == "runner":  # the bench runner's per-step calls; rank 1 fails after step 2
            for i in range(10):
                if rank == 1 and i == 3:
                    hb.fail("injected failure after step 2")
                    results[rank] = "failed"
                    return
                try:
                    hb.step(i, every=4, wait_s=10.0)
                except shard.PeerFailure as err:
                    results[rank] = f"detected at step {i}: {err}"
                    return
            results[rank] = "missed"
        elif mode == "runner_stall":  # rank 1 stops beating after step 2 without a word
            for i in range(10):
                if rank == 1 and i == 3:
                    results[rank] = "stalled"
                    return
                try:
                    hb.step(i, every=4, wait_s=1.0)
                except shard.PeerFailure as err:
                    results[rank] = f"detected at step {i}: {err}"
                    return
            results[rank] = "missed"
        elif mode == "stall":
            hb.beat(0)
            hb.check(0)
            if rank == 1:
                results[rank] = "stalled"  # never beats step 1, never raises
                return
            try:
                hb.check(1, wait_s=1.0)
                results[rank] = "missed"
            except shard.PeerFailure as err:
                results[rank] = f"detected: {err}"
    except RuntimeError as err:
        results[rank] = f"raised: {err}"
    finally:
        if mode == "max":
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    return dict(results)


def test_max_over_ranks_gloo():
    results = _run("max")
    assert results == {0: 11.0, 1: 11.0}


def test_rank_exception_is_detected_by_peer():
    results = _run("raise")
    assert results[1].startswith("raised")
    assert results[0].startswith("detected") and "injected exception" in results[0]


def test_stalled_rank_is_detected_by_peer():
    results = _run("stall")
    assert results[1] == "stalled"
    assert results[0].startswith("detected") and "did not reach step 1" in results[0]


def test_runner_heartbeat_detects_failure_within_a_step():
    results = _run("runner")
    assert results[1] == "failed"
    assert results[0].startswith("detected at step") and "injected failure" in results[0]
    assert int(results[0].split()[3].rstrip(":")) <= 4


def test_runner_heartbeat_detects_silent_stall_at_the_next_progress_check():
    results = _run("runner_stall")
    assert results[1] == "stalled"
    assert results[0] == "detected at step 4: ranks [1] did not reach step 4 within 1.0 s"
