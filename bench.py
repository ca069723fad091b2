"""Benchmark: 1080p frames/s of the RF-DETR-Medium fp32 hot path on B200, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N

A step (ours) is one pass of the whole path over B (default 64) seeded 1920x1080 uint8 frames per GPU — the
512-frame stream of the full-forward config split over 8 GPUs, one step per GPU: the preprocessing
kernel (bit-exact cv2 resize + normalise, written straight into the patch-embedding layout) and the captured
fp32 forward (backbone, projector, top-300 selection, decoder, heads). Frames are independent, so N GPUs each
take their own B frames (weak scaling, no collective on the data path); time is the max over ranks of the
CUDA-event time of K steps. `value` has the frames already resident in HBM (the working set — 120 MB of weights,
~B x 60 MB of activations — is far larger than the 126 MB L2, so no flush is needed); `e2e` runs the same
steps through FastBasketballDetector.detect_stream from pinned host frames, with every step's H2D copy of its
frames and D2H copy of its outputs inside the timed region (pipelined: step i+1's copy-in overlaps step i).
`stream` runs the full-forward config's 512-frame stream as stated: split over the N ranks
(stream.run_sharded_stream), from pinned host frames, with the outputs gathered to the host of rank 0 in stream
order inside the timed region (total work fixed: strong scaling). Both arms preprocess with OpenCV's
fixed-point arithmetic (resize_policy="opencv"), which is bit-exact with the x86-64 cv2.resize the CPU arm calls.

`configs` (rank 0 of a one-GPU run; --no-configs skips it) times the four kernels of configs 1-4 on their own at
each of their batch sizes, with a cold L2 (kernelopt_b200.profile_kernels' workloads).

--impl reference times the reference's CPU path on the host cores instead: cv2.resize + numpy normalisation and
the reference's unfused RF-DETR graph restated in torch-CPU fp32 (the oracle; MLX itself cannot be installed
here), one frame per step, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import numpy as np

H, W = 1080, 1920
METRIC = "1080p frames/s"
WORKLOAD = ("RF-DETR-Medium fp32 inference on seeded 1920x1080 uint8 BGR frames: preprocessing + backbone + "
            "projector + top-300 selection + 4-layer deformable decoder + heads, random-init weights (seed 0)")


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per plain GEMM launch, mean over the 45 plain GEMM
# launches of one 64-frame forward: their algorithmic bytes (x, output, split weight, addend; 450.7 MB per launch)
# times the traffic/algorithmic ratio that one-launch captures of the two largest shapes measured (0.836), each
# from a 32-frame case of one kernel:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum --clock-control none
#       -k regex:gemm_tf32x3 -s 1 -c 1 python -m kernelopt_b200.profile_kernels --kernel gemm --batch 32 \
#       --iters 1 --warmup 1                                    (and --kernel qkv)
# The reads of those captures equal the algorithmic reads; the shortfall is output still in L2 at kernel exit.
GEMM_TRAFFIC_PER_LAUNCH = {64: 376.8e6}


def frames_for(rank: int, n: int) -> np.ndarray:
    rng = np.random.default_rng(1000 + rank)
    return rng.integers(0, 256, (n, H, W, 3), dtype=np.uint8)


def cpu_reference_run(n_frames: int, budget_s: float | None = None):
    """The reference's CPU path, timed: cv2 preprocessing + torch-CPU fp32 unfused forward, one frame per call.
    Returns (frames/s, frames done, threads)."""
    import cv2
    import torch

    from kernelopt_b200.weights import random_weights
    from oracle.model import OracleRFDETR
    from oracle.resize import MEAN, STD

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cv2.setNumThreads(threads)
    model = OracleRFDETR(random_weights(0), torch.float32)
    imgs = frames_for(0, 2)

    def one(img):
        rgb = cv2.cvtColor(cv2.resize(img, (640, 640)), cv2.COLOR_BGR2RGB).astype(np.float32) / 255.
        x = torch.from_numpy(((rgb - MEAN) / STD)[None])
        model(x)

    one(imgs[0])  # warm-up
    done, t0 = 0, time.perf_counter()
    while done < n_frames and (budget_s is None or time.perf_counter() - t0 < budget_s):
        one(imgs[done % 2])
        done += 1
    dt = time.perf_counter() - t0
    return done / dt, done, threads


def run_reference(args, rank: int):
    if rank != 0:
        return
    import cv2
    import torch

    from kernelopt_b200.weights import random_weights
    from oracle.model import OracleRFDETR
    from oracle.resize import MEAN, STD

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cv2.setNumThreads(threads)
    model = OracleRFDETR(random_weights(0), torch.float32)
    imgs = frames_for(0, 2)

    def step(i):
        rgb = cv2.cvtColor(cv2.resize(imgs[i % 2], (640, 640)), cv2.COLOR_BGR2RGB).astype(np.float32) / 255.
        model(torch.from_numpy(((rgb - MEAN) / STD)[None]))

    for i in range(args.warmup):
        step(i)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        step(i)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = args.steps / total
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "frames_per_step": 1, "path": "cv2.resize + numpy normalise + "
                       "torch-CPU fp32 restatement of the reference's unfused graph (MLX unavailable here)"},
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} timed frames of 1920x1080, batch 1"},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "median_ms": 1e3 * statistics.median(times)}
    print(json.dumps(line), flush=True)


def instrumented_step(det, runner_x, items, K):
    """One eager (uncaptured) step with every hot-path kernel call wrapped in CUDA events on its launching
    stream. Returns {kernel: (seconds, work, launches, unit)} and the number of libkernelopt launches."""
    from kernelopt_b200 import _lib
    from kernelopt_b200.benchutil import EventTimer, hold_stream

    timers = {n: EventTimer() for n in ("gemm_tf32x3", "gemm_residual_ln", "attention_tf32x3", "residual_layernorm",
                                         "deform_attn", "preprocess")}
    orig = {n: getattr(K, n) for n in ("linear", "linear_add", "linear_residual_layernorm", "attention",
                                       "residual_layernorm", "deform_attn", "preprocess_batch")}

    def gemm_work(x, pw, *a, **k):
        return 2.0 * (x.numel() // pw.k) * pw.k * pw.n

    def gemm_ln_work(x, pw, *a, **k):
        return 2.0 * (x.numel() // pw.k) * pw.k * pw.n   # the GEMM's flops; the epilogue is memory work

    def attn_work(q, k, v, heads, scale, out=None):
        b, n, w = q.shape
        return 4.0 * b * n * n * w                       # QK^T and PV, all heads

    def ln_work(h, o, *a, **k):
        return 16.0 * h.numel()                          # read h, o; write h_out, y (fp32)

    def deform_work(value, loc, aw, grid_hw, nh, hd, offset=0):
        b, nq = value.shape[0], loc.shape[1]
        npts = loc.shape[-2]
        return 4.0 * b * (grid_hw[0] * grid_hw[1] * nh * hd + nq * nh * npts * 3 + nq * nh * hd)

    def pre_work(items_, lut, dst=640, layout="hwc", out=None):
        return float(sum(img.numel() for img, *_ in items_) + len(items_) * dst * dst * 3 * 4)

    K.linear = timers["gemm_tf32x3"].wrap(orig["linear"], gemm_work)
    K.linear_add = timers["gemm_tf32x3"].wrap(orig["linear_add"], gemm_work)   # the same kernel, + an addend
    K.linear_residual_layernorm = timers["gemm_residual_ln"].wrap(orig["linear_residual_layernorm"], gemm_ln_work)
    K.attention = timers["attention_tf32x3"].wrap(orig["attention"], attn_work)
    K.residual_layernorm = timers["residual_layernorm"].wrap(orig["residual_layernorm"], ln_work)
    K.deform_attn = timers["deform_attn"].wrap(orig["deform_attn"], deform_work)
    K.preprocess_batch = timers["preprocess"].wrap(orig["preprocess_batch"], pre_work)
    before = sum(_lib.launch_count.values())
    try:
        with __import__("torch").cuda.stream(det.stream):
            hold_stream(0.3)   # the host enqueues the whole eager step first: events time GPU work only
            K.preprocess_batch(items, det._lut, 640, "patch16", out=runner_x)
            det.model(runner_x)
        det.stream.synchronize()
    finally:
        for n, f in orig.items():
            setattr(K, n, f)
    launches = sum(_lib.launch_count.values()) - before
    out = {}
    for n, t in timers.items():
        secs, work, cnt = t.total()
        out[n] = (secs, work, cnt, "flop" if n in ("gemm_tf32x3", "gemm_residual_ln", "attention_tf32x3") else "byte")
    return out, launches


# Configs 1-4 (the four kernels at their own sizes): (profile_kernels workload, batch sizes). Config 1's B=3 is the
# three frame sizes in one launch; config 4 samples the decoder's fused [B, 1600, 1024] value layout.
CONFIG_RUNS = (("preprocess", "preprocess", (1, 3, 64)), ("residual_layernorm", "resln", (1, 3, 64)),
               ("linear_gelu_f32", "gemm", (1, 3, 32)), ("deform_attn", "deform_model", (1, 3, 64)))


def config_runs(dev, iters: int = 10) -> dict:
    """CUDA-event time of each kernel at its config's batch sizes, cold L2 (a 256 MB write + read-back before
    every timed launch), the host held off by a spin kernel; median of `iters`."""
    import torch

    from kernelopt_b200.benchutil import hold_stream, measured_peaks
    from kernelopt_b200.profile_kernels import setup

    peaks = measured_peaks()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    res = {}
    for name, kernel, batches in CONFIG_RUNS:
        res[name] = {}
        for b in batches:
            fn, work, unit = setup(kernel, b, dev)
            for _ in range(3):
                fn()
            ts = []
            for _ in range(iters):
                flush.fill_(1.0)
                flush.sum()
                hold_stream(0.002)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) / 1e3)
            t = statistics.median(ts)
            if unit == "flop":
                ach, peak, u = work / t / 1e12, peaks["bf16_tflops"] / 6.0, "TFLOP/s"
            else:
                ach, peak, u = work / t / 1e9, peaks["hbm_gbs"], "GB/s"
            res[name][str(b)] = {"us": t * 1e6, "achieved": ach, "unit": u, "frac": ach / peak}
            del fn
    del flush
    torch.cuda.empty_cache()
    res["note"] = ("configs 1-4 at their batch sizes (1 = 1080p, 3 = 1080p + 720p + 540p, 64 = 64 frames cycling "
                   "those sizes for preprocessing); cold L2, median of %d launches; fractions of the measured HBM "
                   "copy bandwidth or of the 3xTF32 ceiling (measured bf16 / 6)" % iters)
    return res


def run_ours(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from kernelopt_b200 import FastBasketballDetector
    from kernelopt_b200 import kernels as K
    from kernelopt_b200.benchutil import ClockSampler, measured_peaks

    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=300))
    B = args.batch
    # "opencv": the same resize arithmetic as the CPU arm's x86-64 cv2.resize, so both arms see identical inputs
    det = FastBasketballDetector("random:0", warmup_batch_sizes=(), device=dev, resize_policy="opencv")
    host = torch.from_numpy(frames_for(rank, B)).pin_memory()
    frames = host.to(dev)
    mode, xt, yt = det._taps(W, H)
    runner = det._runner(B)
    items = [(frames[i], xt, yt, mode) for i in range(B)]
    stream = det.stream

    def step():
        K.preprocess_batch(items, det._lut, 640, "patch16", out=runner.x)
        runner.run()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident throughput (value) ----
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    secs = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    value = world * B * args.steps / secs
    K.check_device_status(dev)

    # ---- end to end through the public API from pinned host frames (e2e) ----
    # detect_stream pipelines the steps: the H2D copy of step i+1's frames overlaps step i's compute and the D2H
    # of step i's outputs overlaps step i+1. Every step still copies its own frames in and its outputs out.
    for _ in det.detect_stream(host for _ in range(max(2, args.warmup))):
        pass
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in det.detect_stream(host for _ in range(args.steps)):
        pass
    e2e_secs = max_over_ranks(time.perf_counter() - t0)
    e2e = world * B * args.steps / e2e_secs
    barrier()

    # ---- the 512-frame stream split over the ranks, gathered in order on rank 0 (strong scaling) ----
    stream_line = None
    if args.stream_frames > 0:
        from kernelopt_b200.stream import run_sharded_stream, shard_range

        def batch_at(s, e):   # the stream's frames cycle through this rank's B pinned frames
            return host[:e - s]

        # A rank's shard goes through detect_stream in batches of B, or in four smaller ones (at least 8 frames)
        # when the shard is shorter than 4 B: a one-batch shard could not overlap its copy-in with any compute.
        per_rank = -(-args.stream_frames // world)
        sb = B if per_rank >= 4 * B else max(8, per_rank // 4)

        def run_stream():
            if world == 1:
                outs = list(det.detect_stream(batch_at(s, min(s + sb, args.stream_frames))
                                              for s in range(0, args.stream_frames, sb)))
                return np.concatenate([o[0] for o in outs]), np.concatenate([o[1] for o in outs])
            return run_sharded_stream(det.detect_stream, batch_at, args.stream_frames, sb)

        run_stream()                                            # warm-up (and the gather's first use)
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        res = run_stream()
        st_secs = max_over_ranks(time.perf_counter() - t0)
        if rank == 0:
            assert res[0].shape == (args.stream_frames, 300, 4) and res[1].shape == (args.stream_frames, 300, 11)
        # the e2e limiter: pinned host -> device copy rate of one batch, all ranks copying at once
        dev_buf = torch.empty_like(host, device=dev)
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(5):
            dev_buf.copy_(host, non_blocking=True)
        c1.record()
        c1.synchronize()
        h2d_gbs = 5 * host.numel() / (c0.elapsed_time(c1) / 1e3) / 1e9
        h2d_min = -max_over_ranks(-h2d_gbs)
        del dev_buf
        n_mine = len(shard_range(args.stream_frames, rank, world))
        stream_line = {"frames": args.stream_frames, "value": args.stream_frames / st_secs, "unit": "frames/s",
                       "seconds": st_secs, "scaling": "strong", "frames_per_rank": n_mine,
                       "h2d_gbs_per_rank_min": h2d_min, "batch": sb,
                       "path": "run_sharded_stream: detect_stream over the rank's shard in batches of "
                               f"{sb} from pinned host frames, outputs gathered on rank 0 in stream order",
                       "time": "host wall clock from a barrier to the gathered outputs, max over ranks"}
        barrier()

    # ---- latency of one batch of 1 and of 3 frames (config 5's latency runs), frames on the device ----
    latency = {}
    for nb in (1, 3):
        r_nb = det._runner(nb)
        items_nb = [items[i % B] for i in range(nb)]
        ts = []
        with torch.cuda.stream(stream):
            for it in range(25):
                l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                l0.record(stream)
                K.preprocess_batch(items_nb, det._lut, 640, "patch16", out=r_nb.x)
                r_nb.run()
                l1.record(stream)
                l1.synchronize()
                if it >= 5:
                    ts.append(l0.elapsed_time(l1))
        latency[f"frames_{nb}"] = statistics.median(ts)

    # ---- per-kernel timing (CUDA events around each launch, eager) and launch count ----
    per, launches_per_step = instrumented_step(det, runner.x, items, K)
    peaks = measured_peaks()
    tf32x3_peak = peaks["bf16_tflops"] / 6.0   # TF32 runs at half the bf16 rate; 3 products per useful flop
    kernels = {}
    for n, (s, work, cnt, unit) in per.items():
        if cnt == 0:
            continue
        if unit == "flop":
            ach = work / s / 1e12
            kernels[n] = {"launches_per_step": cnt, "ms_per_step": 1e3 * s, "achieved": ach, "unit": "TFLOP/s",
                          "peak": tf32x3_peak, "frac": ach / tf32x3_peak, "bound": "tensor",
                          "tensor_pipe_frac": 3 * ach / (peaks["bf16_tflops"] / 2)}
        else:
            ach = work / s / 1e9
            kernels[n] = {"launches_per_step": cnt, "ms_per_step": 1e3 * s, "achieved": ach, "unit": "GB/s",
                          "peak": peaks["hbm_gbs"], "frac": ach / peaks["hbm_gbs"], "bound": "hbm"}
    dom = max(kernels, key=lambda n: kernels[n]["ms_per_step"])
    dk = kernels[dom]
    roofline = {"kernel": dom, "bound": dk["bound"], "achieved": dk["achieved"], "peak": dk["peak"],
                "unit": dk["unit"], "frac": dk["frac"], "traffic": GEMM_TRAFFIC_PER_LAUNCH.get(B) if dom == "gemm_tf32x3"
                else None, "traffic_unit": "bytes per launch (ncu dram read + write, per-shape one-launch captures scaled to "
                "the step's plain GEMM launches)",
                "peak_source": ("3xTF32 ceiling = measured bf16 dense / 6 (" + peaks["source"] + ")"
                                if dk["bound"] == "tensor" else f"{peaks['source']} HBM copy bandwidth"),
                "step_share_eager": dk["ms_per_step"] / (1e3 * secs / args.steps)}

    line = {"metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "frames_per_step_per_gpu": B, "frame": f"{W}x{H} uint8 BGR",
                       "l2": "inputs + working set > 126 MB L2 (no flush)", "parallelism": f"frame-sharded x{world}",
                       "resize_policy": det.resize_policy},
            "e2e": {"value": e2e, "unit": "frames/s", "h2d_bytes_per_step": int(B * H * W * 3),
                    "d2h_bytes_per_step": int(B * 300 * 15 * 4),
                    "path": "FastBasketballDetector.detect_stream(pinned uint8 frame batches) -> numpy, "
                            "H2D / D2H on a copy stream overlapping the neighbouring steps' compute"},
            "stream": stream_line,
            "gpu_launches": int(launches_per_step * args.steps),
            "roofline": roofline, "kernels": kernels, "clocks": clk.summary(),
            "latency_ms": dict(latency, note="median CUDA-event time of preprocessing + forward for one batch, "
                                             "frames resident on the device")}
    if rank == 0 and world == 1 and not args.no_configs:
        line["configs"] = config_runs(dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fps, n, cores = cpu_reference_run(10_000, budget_s=args.cpu_seconds)
        line["cpu_baseline"] = {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                                "sample": f"{n} frames of 1920x1080, batch 1, cv2 preprocessing + torch-CPU fp32 "
                                          f"unfused forward, ~{args.cpu_seconds:.0f} s budget"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=64,
                    help="frames per step per GPU (64: config 5's 512-frame stream over 8 GPUs)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--stream-frames", type=int, default=512,
                    help="frames of the sharded stream measurement (0 skips it)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-config kernel timings (configs 1-4)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        run_reference(args, rank)
    else:
        run_ours(args, rank, world)


if __name__ == "__main__":
    sys.exit(main())
