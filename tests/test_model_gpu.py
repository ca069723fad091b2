"""Full RF-DETR-Medium forward on the GPU vs the float64 CPU oracle (the reference's unfused graph), and the
reference's own detector tests (batch == single, two instances on two threads: tests/test_fast_rfdetr.py:59-83).

The reference asserts its accuracy bar at batch 1 and 3 (tests/test_fast_rfdetr.py:51-56); the ranking it protects
is the top-300 argsort of model.py:183. On seeded random-init weights that ranking is ill-conditioned for most
frames: neighbouring encoder scores inside the top 300 are often closer than fp32 noise, so no fp32 path (the
reference's own CPU path included) keeps the float64 slot order there. Hence two kinds of test:

  well separated   frames from tests/golden/separated_frames.json (made by make_separated_frames.py), whose
                   float64 top-301 scores are all further apart than twice the GPU's measured score error. The
                   test asserts that precondition, then an identical top-300 index ORDER and, end to end through
                   the public API (raw / raw_batch), max|logit diff| <= 2e-3 and max|box diff| <= 1e-3 — with no
                   condition. B=1 and B=3 (mixed frame sizes) on the default weights, B=1 on weights with
                   non-identity biases, norms, layer scales and proposal mask.
  arbitrary        on the default seeds: the top-300 SET is identical, order mismatches sit between float64 near
                   ties, the decoder on the oracle's memory meets the bars, and the slots matched of 300 (the
                   reference README's measure, README.md:93-104) are reported against float64 and the fp32 CPU port.
"""
from __future__ import annotations

import json
import threading
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle.resize as OR
from kernelopt_b200 import FastBasketballDetector
from kernelopt_b200 import kernels as K
from kernelopt_b200.model import RFDETR
from kernelopt_b200.weights import random_weights
from oracle.model import OracleRFDETR

pytestmark = pytest.mark.gpu

SEPARATED = json.loads((Path(__file__).parent / "golden" / "separated_frames.json").read_text())["frames"]
LOGIT_TOL, BOX_TOL = 2e-3, 1e-3


def frame(seed, h=1080, w=1920):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def rel(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max())


def spec_weights(spec: str):
    name, seed = spec.split(":")
    return random_weights(int(seed), varied=name == "random-varied")


def gpu_scores(model: RFDETR, x_patch: torch.Tensor):
    """(scores [B, 1600], idx [B, 300]) of the GPU path's query selection for PATCH16 input."""
    with torch.no_grad():
        mem = model.projector(model.backbone(x_patch)).reshape(x_patch.shape[0], 1600, 256)
        _, sc, idx = model.select_queries(mem)
    return sc.double().cpu().numpy(), idx.long().cpu().numpy()


def top_gaps(s: np.ndarray, valid: np.ndarray) -> np.ndarray:
    """Consecutive differences of the float64 ranks 1..301, skipping pairs of masked proposals (exact ties)."""
    order = np.argsort(-s, kind="stable")[:301]
    g = -np.diff(s[order])
    return g[~((valid[order[:-1]] == 0) & (valid[order[1:]] == 0))]


CASES = {
    "b1_default": [f for f in SEPARATED if f["weights"] == "random:0" and (f["h"], f["w"]) == (1080, 1920)][:1],
    "b3_default_mixed": [f for f in SEPARATED if f["weights"] == "random:0"][:3],
    "b1_varied": [f for f in SEPARATED if f["weights"] == "random-varied:0"][:1],
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_forward_end_to_end_well_separated(cuda, case):
    """Unconditional end-to-end parity on frames whose ranking fp32 arithmetic cannot reorder."""
    frames = CASES[case]
    assert frames and len({f["weights"] for f in frames}) == 1, "fixture missing for " + case
    if case.startswith("b3"):
        assert len(frames) == 3 and len({(f["h"], f["w"]) for f in frames}) == 3
    spec = frames[0]["weights"]
    w = spec_weights(spec)
    valid = w["proposal_valid"][:, 0]
    imgs = [frame(f["seed"], f["h"], f["w"]) for f in frames]
    det = FastBasketballDetector(spec, warmup_batch_sizes=())
    orc = OracleRFDETR(w, torch.float64)

    # the oracle: preprocessing (reference policy, as the detector's default) + float64 forward, frame by frame
    xs = [torch.from_numpy(OR.preprocess(im))[None] for im in imgs]
    ob, ol, osc, oidx = zip(*(orc(x, return_selection=True) for x in xs))
    ob, ol = torch.cat(ob).numpy(), torch.cat(ol).numpy()
    osc, oidx = torch.cat(osc).numpy(), torch.cat(oidx).numpy()

    # the GPU's own score error on exactly the detector's preprocessed input, and the order it selects
    with torch.cuda.device(det.device), torch.cuda.stream(det.stream):
        patches = torch.stack([det._preprocess(im).reshape(40, 16, 40, 16, 3).permute(0, 2, 1, 3, 4)
                               .reshape(1600, 768) for im in imgs]).contiguous()
        gsc, gidx = gpu_scores(det.model, patches)
    det.stream.synchronize()
    for k, f in enumerate(frames):
        err = float(np.abs(gsc[k] - osc[k]).max())
        gap = float(top_gaps(osc[k], valid).min())
        assert gap == pytest.approx(f["min_gap"], rel=1e-6), "fixture and oracle disagree"
        # precondition of an order-preserving path: every gap is more than twice the score error
        assert 2 * err < gap, f"frame {f['seed']}: GPU score error {err:.2e} vs smallest gap {gap:.2e}"
        assert np.array_equal(gidx[k], oidx[k]), f"frame {f['seed']}: top-300 order differs"

    # end to end through the public API (captured graph, batched preprocessing)
    gb, gl = det.raw_batch(imgs) if len(imgs) > 1 else det.raw(imgs[0])
    dl, db = float(np.abs(gl - ol).max()), float(np.abs(gb - ob).max())
    assert dl <= LOGIT_TOL, f"max logit diff {dl:.2e}"
    assert db <= BOX_TOL, f"max box diff {db:.2e}"
    K.check_device_status()


def test_separated_fixture_covers_every_case():
    """The well-separated cases cannot silently shrink: B=1, B=3 of three sizes, and the varied weights."""
    assert len(CASES["b1_default"]) == 1 and len(CASES["b3_default_mixed"]) == 3 and len(CASES["b1_varied"]) == 1
    for f in SEPARATED:
        assert f["min_gap"] > 2 * f["fp32_oracle_score_error"]


@pytest.fixture(scope="module")
def setup(cuda):
    w = random_weights(0)
    return w, RFDETR(w, cuda), OracleRFDETR(w, torch.float64), OracleRFDETR(w, torch.float32)


def slots_matched(a: np.ndarray, b: np.ndarray) -> int:
    return int((a == b).sum())


@pytest.mark.parametrize("seed", [1, 2])
def test_forward_arbitrary_frames_staged(setup, cuda, seed):
    """Frames with near-tied scores: identical top-300 set, order swaps only between float64 near-ties, the decoder
    on the same memory within the bars, and the slots matched of 300 reported (pytest -s prints them)."""
    _, model, orc, orc32 = setup
    x = torch.from_numpy(OR.preprocess(frame(seed)))[None]
    xp = x.to(cuda).reshape(1, 40, 16, 40, 16, 3).permute(0, 1, 3, 2, 4, 5).reshape(1, 1600, 768).contiguous()
    with torch.no_grad():
        mem_g = model.projector(model.backbone(xp)).reshape(1, 1600, 256)
        mem_o = orc.projector(orc.backbone(x.double())).reshape(1, 1600, 256)
        assert rel(mem_g, mem_o) <= 1e-4, rel(mem_g, mem_o)

        ref_g, sc_g, idx_g = model.select_queries(mem_g)
        ref_o, sc_o, idx_o = orc.select_queries(mem_o)
        _, sc_32, idx_32 = orc32.select_queries(orc32.projector(orc32.backbone(x.float())).reshape(1, 1600, 256))
        score_err = float((sc_g.double().cpu() - sc_o).abs().max())
        assert set(idx_g[0].tolist()) == set(idx_o[0].tolist()), "top-300 set differs"
        ig, io, i32 = idx_g[0].cpu().numpy(), idx_o[0].numpy(), idx_32[0].numpy()
        s = sc_o[0].numpy()
        for k in np.nonzero(ig != io)[0]:
            # a mismatch must sit inside a run of float64 near-ties
            assert abs(s[ig[k]] - s[io[k]]) <= 80 * score_err, (k, s[ig[k]], s[io[k]], score_err)
        print(f"\n[slots matched of 300] seed {seed}: GPU vs float64 {slots_matched(ig, io)}, "
              f"fp32 CPU port vs float64 {slots_matched(i32, io)}, GPU vs fp32 CPU port {slots_matched(ig, i32)}; "
              f"GPU score error {score_err:.2e}, fp32 port score error "
              f"{float((sc_32.double() - sc_o).abs().max()):.2e}")
        assert slots_matched(ig, io) >= 250

        hs_g = model.decoder(mem_o.float().to(cuda), ref_o.float().to(cuda))
        hs_o = orc.decoder(mem_o, ref_o)
        lg = model.class_embed(hs_g)
        lo = orc.lin(hs_o, "class_embed")
        assert float((lg.double().cpu() - lo).abs().max()) <= LOGIT_TOL
        dg = model._mlp3(hs_g, model.bbox_embed)
        do = orc.mlp3(hs_o, "bbox_embed")
        r = ref_o.float().to(cuda)
        bg = torch.cat([dg[..., :2] * r[..., 2:] + r[..., :2], torch.exp(dg[..., 2:]) * r[..., 2:]], -1)
        bo = torch.cat([do[..., :2] * ref_o[..., 2:] + ref_o[..., :2], torch.exp(do[..., 2:]) * ref_o[..., 2:]], -1)
        assert float((bg.double().cpu() - bo).abs().max()) <= BOX_TOL
    torch.cuda.synchronize()
    K.check_device_status()


@pytest.fixture(scope="module")
def det(cuda):
    return FastBasketballDetector("random:0", warmup_batch_sizes=(1, 3))


def test_detector_raw_shapes_and_errors(det):
    b, lg = det.raw(frame(5))
    assert b.shape == (1, 300, 4) and lg.shape == (1, 300, 11)
    assert b.dtype == np.float32 and lg.dtype == np.float32
    with pytest.raises(ValueError):
        det.raw_batch([])
    with pytest.raises(ValueError):
        det.raw_batch([frame(1)] * 4)
    with pytest.raises(ValueError):
        det.raw(frame(1).astype(np.float32))
    with pytest.raises(ValueError):
        FastBasketballDetector("random:0", precision="fp16", warmup_batch_sizes=())


def test_preprocess_bitwise_identical(det):
    """The reference's test_gpu_preprocess_bitwise_identical (tests/test_fast_rfdetr.py:46-49), on seeded frames."""
    for img in (frame(11), frame(12, 1080, 1152), frame(13, 720, 1280)):
        g = det._preprocess(img).cpu().numpy()
        assert np.array_equal(g.view(np.uint32), OR.preprocess(img).view(np.uint32))


def test_batch_matches_single(det):
    imgs = [frame(21), frame(22, 1080, 1152), frame(23, 1080, 1152)]
    bb, bl = det.raw_batch(imgs)
    for k, im in enumerate(imgs):
        sb, sl = det.raw(im)
        assert np.abs(bb[k] - sb[0]).max() < 1e-3 and np.abs(bl[k] - sl[0]).max() < 1e-2


def test_bench_batch_graph_matches_batch_one(det):
    """The 64-frame captured graph the benchmark times, against batch-1 runs of the same frames (the bench's own
    seeded 1080p noise frames). The graph replays exactly the eager 64-frame forward (bitwise). Batch size may
    change GEMM tiles and LayerNorm CTA layouts, so scores may move in the last bits; where a frame's top-301
    gaps exceed twice that movement the slot order is provably the same, and there the outputs must agree
    within the end-to-end bars. Elsewhere the top-300 sets must agree up to near-ties at rank 300."""
    model = det.model
    frames = np.random.default_rng(1000).integers(0, 256, (64, 1080, 1920, 3), dtype=np.uint8)
    gb, gl = det.detect_frames(torch.from_numpy(frames).pin_memory())      # the 64-frame graph
    x64 = det._runner(64).x.clone()                                         # its preprocessed input
    with torch.cuda.device(det.device), torch.cuda.stream(det.stream), torch.no_grad():
        eb, el = model(x64)
        assert np.array_equal(eb.cpu().numpy(), gb) and np.array_equal(el.cpu().numpy(), gl), \
            "graph replay differs from the eager forward"
        s64, i64 = gpu_scores(model, x64)
        stable = 0
        for k in range(64):
            s1, i1 = gpu_scores(model, x64[k:k + 1])
            move = float(np.abs(s64[k] - s1[0]).max())
            assert move <= 2e-5, f"frame {k}: batch size moved scores by {move:.2e}"
            gaps = top_gaps(s1[0], np.ones(1600))
            if gaps.min() > 2 * move:
                stable += 1
                assert np.array_equal(i64[k], i1[0]), f"frame {k}: order differs on a stable ranking"
                b1, l1 = model(x64[k:k + 1])
                assert float((b1[0].cpu() - torch.from_numpy(gb[k])).abs().max()) <= BOX_TOL
                assert float((l1[0].cpu() - torch.from_numpy(gl[k])).abs().max()) <= LOGIT_TOL
            else:
                d = set(i64[k].tolist()) ^ set(i1[0].tolist())
                top = np.sort(s1[0])[::-1]
                assert all(abs(s1[0][j] - top[299]) <= 4 * move for j in d), f"frame {k}: top-300 sets differ"
    torch.cuda.synchronize()
    print(f"\n[64-frame graph vs batch 1] {stable}/64 frames with a provably stable ranking matched within the bars")
    assert stable >= 8


def test_two_instances_two_threads(det):
    other = FastBasketballDetector("random:0")
    imgs = [frame(30 + i) for i in range(4)]
    expected = [det.raw(im) for im in imgs]
    errors = []

    def work(d, off):
        for k in range(12):
            i = (k + off) % len(imgs)
            b, lg = d.raw(imgs[i])
            if not (np.array_equal(b, expected[i][0]) and np.array_equal(lg, expected[i][1])):
                errors.append(i)

    th = [threading.Thread(target=work, args=(d, o)) for d, o in ((det, 0), (other, 2))]
    [t.start() for t in th]
    [t.join() for t in th]
    assert not errors


def test_detect_stream_matches_detect_frames(det):
    """The pipelined stream API gives, batch for batch, exactly what detect_frames gives on the same frames —
    including when batches alternate between two pinned host buffers and the slots are reused."""
    bufs = [torch.from_numpy(np.stack([frame(40 + 3 * j + i) for i in range(3)])).pin_memory() for j in range(2)]
    expected = [det.detect_frames(b) for b in bufs]
    order = [0, 1, 1, 0, 1, 0, 0]
    got = list(det.detect_stream(bufs[j] for j in order))
    assert len(got) == len(order)
    for (gb, gl), j in zip(got, order):
        assert np.array_equal(gb, expected[j][0]) and np.array_equal(gl, expected[j][1])
    with pytest.raises(ValueError):
        list(det.detect_stream([bufs[0], bufs[0][:2]]))


def test_detect_stream_stopped_early_leaves_no_work_behind(det):
    """A consumer that breaks out after the first batch: the generator's clean-up waits for the queued copies and
    compute, so the slot buffers it frees cannot be handed to new work while still in use."""
    bufs = [torch.from_numpy(np.stack([frame(60 + 3 * j + i) for i in range(3)])).pin_memory() for j in range(3)]
    expected = det.detect_frames(bufs[0])
    gen = det.detect_stream(iter(bufs))
    first = next(gen)
    gen.close()                                      # runs the generator's finally block
    assert np.array_equal(first[0], expected[0]) and np.array_equal(first[1], expected[1])
    junk = [torch.full((1 << 22,), 7, dtype=torch.uint8, device=det.device) for _ in range(8)]
    torch.cuda.synchronize()
    del junk
    again = det.detect_frames(bufs[0])
    assert np.array_equal(again[0], expected[0]) and np.array_equal(again[1], expected[1])
