"""Frame streams over several GPUs. Frames are independent, so there is no collective on the data path: each GPU
runs whole frames through its own detector, and only the small outputs (300 x 15 floats per frame) travel back.

Two runners:
  * shard_range / run_sharded / run_sharded_stream: one process per GPU (torch.distributed, launched by
    torchrun). Rank r takes a contiguous shard of the stream, produces its frames itself (decoder or generator,
    frame index -> image), and rank 0 gathers the outputs in stream order (an object gather of host arrays; the
    process group may be nccl or gloo). run_sharded calls a batch detector per batch; run_sharded_stream feeds
    the shard as uint8 frame batches to a pipelined detector (FastBasketballDetector.detect_stream), so copies
    in and out overlap the compute of the neighbouring batches.
  * QueueRunner: one process driving several GPUs from worker threads that pull batches from a shared queue.
    If a worker fails (an exception from its detector: a launch error, a device-side timeout reported by
    check_device_status, a lost device), its batch goes back on the queue for the surviving workers and the
    worker retires; the stream completes as long as one worker is alive.
"""
from __future__ import annotations

import queue
import threading
from collections.abc import Callable, Sequence

import numpy as np

DetectFn = Callable[[list[np.ndarray]], tuple[np.ndarray, np.ndarray]]


def shard_range(n_frames: int, rank: int, world: int) -> range:
    """Contiguous shard of frame indices for `rank` (sizes differ by at most one)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(n_frames, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def run_sharded(detect: DetectFn, frame_at: Callable[[int], np.ndarray], n_frames: int, batch: int,
                group=None):
    """Runs this rank's shard in batches and gathers (boxes [n,300,4], logits [n,300,11]) on rank 0 in stream
    order; other ranks return None."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    idx = shard_range(n_frames, rank, world)
    boxes, logits = [], []
    for s in range(idx.start, idx.stop, batch):
        b, lg = detect([frame_at(i) for i in range(s, min(s + batch, idx.stop))])
        boxes.append(b)
        logits.append(lg)
    return _gather(idx.start, boxes, logits, rank, world, group)


def run_sharded_stream(detect_stream: Callable, batch_at: Callable, n_frames: int, batch: int, group=None):
    """run_sharded for a pipelined detector. detect_stream(iterable of frame batches) yields (boxes, logits) per
    batch in order; batch_at(start, stop) returns the frames [start, stop) of the stream as one batch (e.g. a
    uint8 tensor [stop - start, H, W, 3] in pinned host memory). Full batches go through one detect_stream
    pass and a shorter last batch through a second one (a pipelined stream keeps one batch shape). Gathers
    (boxes [n,300,4], logits [n,300,11]) on rank 0 in stream order; other ranks return None."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    idx = shard_range(n_frames, rank, world)
    full = [(s, s + batch) for s in range(idx.start, idx.stop - batch + 1, batch)]
    tail = [(full[-1][1] if full else idx.start, idx.stop)]
    boxes, logits = [], []
    for spans in (full, [t for t in tail if t[1] > t[0]]):
        for b, lg in detect_stream(batch_at(s, e) for s, e in spans):
            boxes.append(b)
            logits.append(lg)
    return _gather(idx.start, boxes, logits, rank, world, group)


def _gather(start: int, boxes: list, logits: list, rank: int, world: int, group):
    import torch.distributed as dist
    mine = (start, np.concatenate(boxes) if boxes else np.zeros((0, 300, 4), np.float32),
            np.concatenate(logits) if logits else np.zeros((0, 300, 11), np.float32))
    parts = [None] * world if rank == 0 else None
    dist.gather_object(mine, parts, dst=0, group=group)
    if rank != 0:
        return None
    parts.sort(key=lambda p: p[0])
    return np.concatenate([p[1] for p in parts]), np.concatenate([p[2] for p in parts])


class WorkerFailed(RuntimeError):
    pass


class QueueRunner:
    """Dynamic multi-GPU stream runner with re-queueing of failed batches (see module doc)."""

    def __init__(self, detectors: Sequence[DetectFn], batch: int):
        if not detectors:
            raise ValueError("need at least one detector")
        self.detectors = list(detectors)
        self.batch = batch
        self.failures: list[tuple[int, BaseException]] = []

    def run(self, frame_at: Callable[[int], np.ndarray], n_frames: int):
        todo: queue.Queue = queue.Queue()
        for s in range(0, n_frames, self.batch):
            todo.put((s, min(s + self.batch, n_frames)))
        n_batches = todo.qsize()
        results: dict[int, tuple[np.ndarray, np.ndarray]] = {}
        lock = threading.Lock()
        alive = [True] * len(self.detectors)
        done = threading.Event()

        def worker(w: int):
            det = self.detectors[w]
            while not done.is_set():
                try:
                    s, e = todo.get(timeout=0.05)
                except queue.Empty:
                    with lock:
                        if len(results) == n_batches:
                            done.set()
                    continue
                try:
                    out = det([frame_at(i) for i in range(s, e)])
                except BaseException as exc:  # noqa: BLE001 - any failure retires the worker
                    todo.put((s, e))
                    with lock:
                        self.failures.append((w, exc))
                        alive[w] = False
                        if not any(alive):
                            done.set()
                    return
                with lock:
                    results[s] = out
                    if len(results) == n_batches:
                        done.set()

        threads = [threading.Thread(target=worker, args=(w,), daemon=True) for w in range(len(self.detectors))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if len(results) != n_batches:
            raise WorkerFailed(f"all workers failed; last error: {self.failures[-1][1]!r}")
        order = sorted(results)
        return (np.concatenate([results[s][0] for s in order]), np.concatenate([results[s][1] for s in order]))
