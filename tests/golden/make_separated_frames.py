"""Finds seeded frames whose top-300 query ranking is well conditioned, for the unconditional full-forward test.

On random-init weights the encoder scores of neighbouring ranks inside the top 300 are often closer than fp32
noise (~2e-6), so no fp32 implementation — the reference's own CPU path included — reproduces the float64 slot
order on an arbitrary frame. This script screens `--limit` seeded frames per (weights, frame size) with the
float32 CPU oracle, confirms the best few in float64, and keeps the frame whose smallest float64 gap between
consecutive top-301 scores is the largest multiple of the float32 oracle's measured score error (it must be at
least `--margin`). Ties between proposals that the mask zeroes are exact by construction and skipped. On those
frames the identical index order follows from a measured score error below half the smallest gap, so the test
asserts it, and the end-to-end logit bar, without conditions.

Measured on 30 frames per weight set: the fraction of frames whose every gap clears 20x the float32 error
(4e-5) is ~3e-7, 10x about 6e-4, 5x about 4e-2 — so the margin is a best-of-N search, not a fixed 20x.

    python tests/golden/make_separated_frames.py [--margin 5] [--limit 600] [--out tests/golden/separated_frames.json]

The frames are `numpy.random.default_rng(seed).integers(0, 256, (h, w, 3), uint8)`, preprocessed by the
oracle's table model under the reference policy. Test infrastructure only.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle.resize as OR  # noqa: E402
from kernelopt_b200.weights import random_weights  # noqa: E402
from oracle.model import OracleRFDETR  # noqa: E402

# (weights, frame size h x w, how many frames) — B=1 and B=3 (mixed sizes) on the default weights, B=1 on the
# varied ones
WANT = [("random:0", (1080, 1920), 1), ("random:0", (720, 1280), 1), ("random:0", (540, 960), 1),
        ("random-varied:0", (1080, 1920), 1)]


def weights(spec: str):
    name, seed = spec.split(":")
    return random_weights(int(seed), varied=name == "random-varied")


def frame(seed: int, h: int, w: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def scores(model: OracleRFDETR, x: torch.Tensor) -> np.ndarray:
    with torch.no_grad():
        mem = model.projector(model.backbone(x.to(model.dtype))).reshape(1, 1600, 256)
        _, s, _ = model.select_queries(mem)
    return s[0].double().numpy()


def top_gaps(s: np.ndarray, valid: np.ndarray) -> np.ndarray:
    """Differences between consecutive scores of ranks 1..301 (stable descending order), skipping pairs of
    masked proposals (their inputs are identical zeros, so their scores tie exactly in every implementation)."""
    order = np.argsort(-s, kind="stable")[:301]
    g = -np.diff(s[order])
    both_masked = (valid[order[:-1]] == 0) & (valid[order[1:]] == 0)
    return g[~both_masked]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--margin", type=float, default=5.0, help="least accepted min gap / float32 score error")
    ap.add_argument("--start", type=int, default=1000)
    ap.add_argument("--limit", type=int, default=600, help="seeds screened per (weights, size)")
    ap.add_argument("--confirm", type=int, default=6, help="best float32 candidates confirmed in float64")
    ap.add_argument("--out", default=str(Path(__file__).with_name("separated_frames.json")))
    args = ap.parse_args()
    found = []
    for spec, (h, w), count in WANT:
        wts = weights(spec)
        valid = wts["proposal_valid"][:, 0]
        o32, o64 = OracleRFDETR(wts, torch.float32), OracleRFDETR(wts, torch.float64)
        t0 = time.time()
        screened = []
        for seed in range(args.start, args.start + args.limit):
            s32 = scores(o32, OR_x(seed, h, w))
            screened.append((float(top_gaps(s32, valid).min()), seed, s32))
            screened.sort(key=lambda t: -t[0])
            del screened[args.confirm:]
        best = []
        for _, seed, s32 in screened:
            s64 = scores(o64, OR_x(seed, h, w))
            err32 = float(np.abs(s32 - s64).max())
            gaps = top_gaps(s64, valid)
            print(f"{spec} {h}x{w} seed {seed}: min gap {gaps.min():.3e}, fp32 error {err32:.3e}, "
                  f"margin {gaps.min() / err32:.1f}", flush=True)
            best.append(dict(weights=spec, seed=seed, h=h, w=w, min_gap=float(gaps.min()),
                             mean_gap=float(gaps.mean()), fp32_oracle_score_error=err32,
                             margin=float(gaps.min() / err32), screened=args.limit))
        best.sort(key=lambda d: -d["margin"])
        best = [d for d in best if d["margin"] >= args.margin][:count]
        print(f"{spec} {h}x{w}: {len(best)} kept in {time.time() - t0:.0f} s", flush=True)
        if len(best) < count:
            raise SystemExit(f"no frame with margin >= {args.margin} for {spec} {h}x{w} in {args.limit} seeds")
        found += best
    Path(args.out).write_text(json.dumps(dict(
        generator="tests/golden/make_separated_frames.py", frame="default_rng(seed).integers(0, 256, (h, w, 3))",
        preprocess="oracle.resize.preprocess (reference policy)", frames=found), indent=1) + "\n")
    print("wrote", args.out)


def OR_x(seed: int, h: int, w: int) -> torch.Tensor:
    return torch.from_numpy(OR.preprocess(frame(seed, h, w)))[None]


if __name__ == "__main__":
    main()
