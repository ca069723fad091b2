"""Runs one hot-path kernel at the benchmark configurations and reports its CUDA-event time and roofline.

    python -m kernelopt_b200.profile_kernels --kernel gemm --batch 32 [--iters 20] [--warmup 3]

Kernels and workloads (per frame of batch B; the algorithmic traffic or flops counted for the roofline):
  preprocess  B frames, sizes cycling 1920x1080 / 1280x720 / 960x540 (B=1: 1080p only), seeded noise,
              PATCH16 output; bytes = H*W*3 read + 640*640*3*4 written per frame (--policy picks the tables)
  preprocess_1080p  the benchmark's frames: B seeded 1920x1080 noise frames, PATCH16 output
  resln       rows = B*1600, C = 384, x/residual ~ N(0,1); bytes = 4 * rows * 384 * 4
  gemm        GELU(A @ W + b), A [B*1600, 384] ~ N(0,1), W [384, 1536] ~ N(0, 0.02^2); flops = 2*M*384*1536
  deform      value [B,1600,16,16], loc U[-0.05,1.05], softmax aw; bytes = 2,060,800 per frame
  deform_model the decoder's layout: value [B,1600,1024] (four layers' projections side by side), layer 1's
              columns [256, 512); the same bytes per frame (the layer's slice of the map is what is sampled)
  attn        the backbone's global attention: B frames x 1604 tokens x 6 heads x 64, q/k/v column slices of
              one [B, 1604, 1152] projection ~ N(0,1); flops = 4 * B * 6 * 1604^2 * 64
  attn_win    the windowed attention: 4B windows x 401 tokens x 6 heads x 64; flops = 4 * 4B * 6 * 401^2 * 64
  outproj_ln  the out-projection + bias, * layer scale, + residual, LayerNorm in one kernel: x [B*1604, 384],
              W [384, 384]; flops = 2*M*384*384 (outproj_unfused: the GEMM, then the residual + LN kernel)
  fc2_ln      the same for fc2: x [B*1604, 1536], W [1536, 384] (fc2_unfused likewise)
  qkv         the fused QKV projection: x [B*1604, 384] @ W [384, 1152] + b; flops = 2*M*384*1152
  conv3x3_ln  the projector's bottleneck conv: x NHWC [B, 40, 40, 128], 3x3 -> 128 channels, LayerNorm + SiLU
              (implicit GEMM); flops = 2*M*1152*128
  cv1_ln      the projector's first 1x1 conv: x [B*1600, 1536] -> 256 channels, LayerNorm + SiLU; flops =
              2*M*1536*256
Each timed iteration is preceded, outside the events, by a write and a read-back of a 256 MB buffer (larger
than the 126 MB L2): every launch starts with a cold L2 that holds no dirty lines of the flush (their write-back
would otherwise be charged to the timed kernel), and a short spin kernel holds the stream while the host enqueues the
launch, so the events time the GPU's work alone. One JSON line per run. Under ncu, use --iters 1-3.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import kernels as K
from .benchutil import hold_stream, measured_peaks
from .resize_tables import tables

SIZES = [(1080, 1920), (720, 1280), (540, 960)]


def setup(kernel: str, b: int, dev, policy: str = "reference"):
    g = torch.Generator(device="cpu").manual_seed(0)
    if kernel in ("preprocess", "preprocess_1080p"):
        rng = np.random.default_rng(0)
        sizes = [SIZES[0]] * b if b == 1 or kernel == "preprocess_1080p" else [SIZES[i % 3] for i in range(b)]
        lut = (np.arange(256, dtype=np.float32)[:, None] / 255. - np.asarray([.485, .456, .406], np.float32)) \
            / np.asarray([.229, .224, .225], np.float32)
        lut_d = torch.from_numpy(np.ascontiguousarray(lut.T)).to(dev)
        items = []
        for h, w in sizes:
            mode, xt, yt = tables(w, h, policy=policy)
            img = torch.from_numpy(rng.integers(0, 256, (h, w, 3), dtype=np.uint8)).to(dev)
            items.append((img, torch.from_numpy(np.array(xt)).to(dev), torch.from_numpy(np.array(yt)).to(dev), mode))
        out = torch.empty((b, 1600, 768), device=dev)
        work = float(sum(h * w * 3 for h, w in sizes) + b * 640 * 640 * 3 * 4)
        return (lambda: K.preprocess_batch(items, lut_d, 640, "patch16", out=out)), work, "byte"
    if kernel == "resln":
        rows = b * 1600
        h = torch.randn(rows, 384, generator=g).to(dev)
        o = torch.randn(rows, 384, generator=g).to(dev)
        gamma = (1 + 0.1 * torch.randn(384, generator=g)).to(dev)
        beta = (0.1 * torch.randn(384, generator=g)).to(dev)
        return (lambda: K.residual_layernorm(h, o, None, None, gamma, beta, 1e-6)), 16.0 * rows * 384, "byte"
    if kernel == "gemm":
        m = b * 1600
        a = torch.randn(m, 384, generator=g).to(dev)
        w = (0.02 * torch.randn(384, 1536, generator=g)).to(dev)
        bias = (0.01 * torch.randn(1536, generator=g)).to(dev)
        pw = K.pack_weight(w, bias)
        return (lambda: K.linear(a, pw, "gelu")), 2.0 * m * 384 * 1536, "flop"
    if kernel in ("outproj_ln", "outproj_unfused", "fc2_ln", "fc2_unfused"):
        m, k = b * 1604, (384 if kernel.startswith("outproj") else 1536)
        x = torch.randn(m, k, generator=g).to(dev)
        w = (torch.randn(k, 384, generator=g) / k ** 0.5).to(dev)
        bias = (0.1 * torch.randn(384, generator=g)).to(dev)
        scale = (1 + 0.1 * torch.randn(384, generator=g)).to(dev)
        h = torch.randn(m, 384, generator=g).to(dev)
        gamma = (1 + 0.1 * torch.randn(384, generator=g)).to(dev)
        beta = (0.1 * torch.randn(384, generator=g)).to(dev)
        if kernel.endswith("_ln"):
            pw = K.pack_weight(w, bias)
            fn = lambda: K.linear_residual_layernorm(x, pw, gamma, beta, 1e-6, resid=h, scale=scale)  # noqa: E731
        else:
            pw = K.pack_weight(w)
            fn = lambda: K.residual_layernorm(h, K.linear(x, pw), bias, scale, gamma, beta, 1e-6)  # noqa: E731
        return fn, 2.0 * m * k * 384, "flop"
    if kernel in ("conv3x3_ln", "cv1_ln"):
        cin, cout, k = (128, 128, 9 * 128) if kernel == "conv3x3_ln" else (1536, 256, 1536)
        x = torch.randn(b, 40, 40, cin, generator=g).to(dev)
        w = (torch.randn(k, cout, generator=g) / k ** 0.5).to(dev)
        gamma = (1 + 0.1 * torch.randn(cout, generator=g)).to(dev)
        beta = (0.1 * torch.randn(cout, generator=g)).to(dev)
        pw = K.pack_weight(w)
        if kernel == "conv3x3_ln":
            fn = lambda: K.conv3x3_layernorm(x, pw, gamma, beta, 1e-6, "silu")  # noqa: E731
        else:
            fn = lambda: K.linear_residual_layernorm(x.reshape(-1, cin), pw, gamma, beta, 1e-6, act="silu",  # noqa: E731
                                                     write_h=False)
        return fn, 2.0 * b * 1600 * k * cout, "flop"
    if kernel == "qkv":
        m = b * 1604
        a = torch.randn(m, 384, generator=g).to(dev)
        w = (torch.randn(384, 1152, generator=g) / 384 ** 0.5).to(dev)
        bias = (0.01 * torch.randn(1152, generator=g)).to(dev)
        pw = K.pack_weight(w, bias)
        return (lambda: K.linear(a, pw)), 2.0 * m * 384 * 1152, "flop"
    if kernel == "deform":
        value = torch.randn(b, 1600, 256, generator=g).to(dev)
        loc = (torch.rand(b, 300, 16, 2, 2, generator=g) * 1.1 - 0.05).to(dev)
        aw = torch.softmax(torch.randn(b, 300, 16, 2, generator=g), -1).to(dev)
        return (lambda: K.deform_attn(value, loc, aw, (40, 40), 16, 16)), 2060800.0 * b, "byte"
    if kernel == "deform_model":
        value = torch.randn(b, 1600, 1024, generator=g).to(dev)
        loc = (torch.rand(b, 300, 16, 2, 2, generator=g) * 1.1 - 0.05).to(dev)
        aw = torch.softmax(torch.randn(b, 300, 16, 2, generator=g), -1).to(dev)
        return (lambda: K.deform_attn(value, loc, aw, (40, 40), 16, 16, offset=256)), 2060800.0 * b, "byte"
    if kernel in ("attn", "attn_win"):
        nb, n = (b, 1604) if kernel == "attn" else (4 * b, 401)
        qkv = torch.randn(nb, n, 1152, generator=g).to(dev)
        q, k, v = qkv[..., :384], qkv[..., 384:768], qkv[..., 768:]
        return (lambda: K.attention(q, k, v, 6, 0.125)), 4.0 * nb * 6 * n * n * 64, "flop"
    raise ValueError(kernel)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True, choices=["preprocess", "preprocess_1080p", "resln", "gemm", "deform", "deform_model",
                                                             "attn", "attn_win",
                                                             "outproj_ln", "outproj_unfused", "fc2_ln", "fc2_unfused", "qkv",
                                                             "conv3x3_ln", "cv1_ln"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--policy", choices=["reference", "opencv"], default="reference",
                    help="resize tables of the preprocess kernels")
    args = ap.parse_args()
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda:0")
    fn, work, unit = setup(args.kernel, args.batch, dev, args.policy)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)   # 256 MB > L2
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.iters):
        flush.fill_(1.0)
        flush.sum()          # read it back: the fill's dirty lines are written back before the timed launch
        hold_stream(0.002)   # the host's launch overhead stays outside the events
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    K.check_device_status(dev)
    t = float(np.median(times))
    peaks = measured_peaks()
    if unit == "flop":
        ach, peak, u = work / t / 1e12, peaks["bf16_tflops"] / 6.0, "TFLOP/s"
    else:
        ach, peak, u = work / t / 1e9, peaks["hbm_gbs"], "GB/s"
    print(json.dumps({"kernel": args.kernel, "batch": args.batch, "median_us": t * 1e6, "min_us": min(times) * 1e6,
                      "achieved": ach, "unit": u, "peak": peak, "frac": ach / peak,
                      "peak_source": peaks["source"] + (" bf16/6 (3xTF32 ceiling)" if unit == "flop" else " HBM"),
                      "work_per_launch": work, "iters": args.iters}), flush=True)


if __name__ == "__main__":
    main()
