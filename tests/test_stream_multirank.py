"""Frame-sharded stream runners on the host (CPU): 2 gloo ranks with fake detectors, and the in-process queue
runner with a worker that fails mid-stream (its batch is re-queued to the surviving worker)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from kernelopt_b200.stream import QueueRunner, WorkerFailed, run_sharded, run_sharded_stream, shard_range


def fake_frame(i: int) -> np.ndarray:
    return np.full((4, 6, 3), i % 251, np.uint8)


def fake_detect(frames):
    ids = np.asarray([int(f[0, 0, 0]) for f in frames], np.float32)
    boxes = np.broadcast_to(ids[:, None, None], (len(frames), 300, 4)).copy()
    logits = np.broadcast_to(-ids[:, None, None], (len(frames), 300, 11)).copy()
    return boxes, logits


def test_shard_range_covers_stream():
    for n, world in [(512, 8), (512, 3), (7, 4), (0, 2)]:
        shards = [shard_range(n, r, world) for r in range(world)]
        flat = [i for s in shards for i in s]
        assert flat == list(range(n))
        assert max(len(s) for s in shards) - min(len(s) for s in shards) <= 1


def fake_detect_stream(batches):
    """A pipelined detector's contract: one (boxes, logits) per batch, in order, every batch of one shape."""
    shape = None
    for frames in batches:
        shape = shape or frames.shape
        assert frames.shape == shape, "a pipelined stream keeps one batch shape"
        yield fake_detect(list(frames))


def _rank_main(rank, world, port, n, out_path, pipelined=False):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    if pipelined:
        res = run_sharded_stream(fake_detect_stream, lambda s, e: np.stack([fake_frame(i) for i in range(s, e)]),
                                 n, batch=5)
    else:
        res = run_sharded(fake_detect, fake_frame, n, batch=5)
    if rank == 0:
        np.save(out_path, res[0][:, 0, 0])
    else:
        assert res is None
    dist.destroy_process_group()


def test_run_sharded_two_gloo_ranks(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "ids.npy"
    mp.start_processes(_rank_main, args=(2, port, 23, str(out)), nprocs=2, join=True, start_method="spawn")
    assert np.array_equal(np.load(out), np.arange(23, dtype=np.float32))


@pytest.mark.parametrize("n", [23, 20, 3])
def test_run_sharded_stream_two_gloo_ranks(tmp_path, n):
    """Shards of 12 + 11 frames in batches of 5 (full batches, then a shorter tail through a second pass), shards
    that are whole batches, and shards shorter than one batch: outputs come back on rank 0 in stream order."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "ids.npy"
    mp.start_processes(_rank_main, args=(2, port, n, str(out), True), nprocs=2, join=True, start_method="spawn")
    assert np.array_equal(np.load(out), np.arange(n, dtype=np.float32))


def test_queue_runner_requeues_failed_batch():
    calls = {"n": 0}

    def flaky(frames):
        calls["n"] += 1
        if calls["n"] == 2:
            raise RuntimeError("simulated device failure")
        return fake_detect(frames)

    runner = QueueRunner([flaky, fake_detect], batch=4)
    boxes, logits = runner.run(fake_frame, 30)
    assert np.array_equal(boxes[:, 0, 0], np.arange(30, dtype=np.float32))
    assert np.array_equal(logits[:, 0, 0], -np.arange(30, dtype=np.float32))
    assert len(runner.failures) == 1 and runner.failures[0][0] == 0


def test_queue_runner_all_workers_fail():
    def dead(frames):
        raise RuntimeError("down")

    with pytest.raises(WorkerFailed):
        QueueRunner([dead, dead], batch=4).run(fake_frame, 10)
