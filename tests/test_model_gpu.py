"""Full RF-DETR-Medium forward on the GPU vs the float64 CPU oracle (the reference's unfused graph), and the
reference's own detector tests (batch == single, two instances on two threads: tests/test_fast_rfdetr.py:59-83).

The check is staged because the top-300 ranking on seeded random-init weights is ill-conditioned: consecutive
encoder scores inside the top 300 can be ~1e-7 apart, below ordinary fp32 noise (the reference's own CPU fp32
path already reorders slots against float64). So:
  memory      projector output, relative max-norm error <= 1e-4
  selection   the top-300 index SET is identical; the ORDER is identical except for swaps of neighbours whose
              float64 scores are closer than 20x the measured max score error (reported as near-ties)
  decoder     given the same memory and reference points, max|logit diff| <= 2e-3 and max|box diff| <= 1e-3
  end to end  when the order is identical, max|logit diff| <= 2e-3
"""
from __future__ import annotations

import threading

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


@pytest.fixture(scope="module")
def setup(cuda):
    w = random_weights(0)
    return w, RFDETR(w, cuda), OracleRFDETR(w, torch.float64)


def frame(seed, h=1080, w=1920):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def rel(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("seed", [1, 2])
def test_forward_staged_vs_oracle(setup, cuda, seed):
    _, model, orc = setup
    x = torch.from_numpy(OR.preprocess(frame(seed)))[None]
    with torch.no_grad():
        mem_g = model.projector(model.backbone(x.to(cuda).reshape(1, 40, 16, 40, 16, 3).permute(0, 1, 3, 2, 4, 5)
                                               .reshape(1, 1600, 768).contiguous())).reshape(1, 1600, 256)
        mem_o = orc.projector(orc.backbone(x.double())).reshape(1, 1600, 256)
        assert rel(mem_g, mem_o) <= 1e-4, rel(mem_g, mem_o)

        ref_g, sc_g, idx_g = model.select_queries(mem_g)
        ref_o, sc_o, idx_o = orc.select_queries(mem_o)
        score_err = float((sc_g.double().cpu() - sc_o).abs().max())
        assert set(idx_g[0].tolist()) == set(idx_o[0].tolist()), "top-300 set differs"
        ig, io = idx_g[0].cpu().numpy(), idx_o[0].numpy()
        s = sc_o[0].numpy()
        near = 20 * score_err
        for k in np.nonzero(ig != io)[0]:
            # a mismatch must sit inside a run of near-tied float64 scores
            assert abs(s[ig[k]] - s[io[k]]) <= near * 4, (k, s[ig[k]], s[io[k]], score_err)

        hs_g = model.decoder(mem_o.float().to(cuda), ref_o.float().to(cuda))
        hs_o = orc.decoder(mem_o, ref_o)
        lg = model.class_embed(hs_g)
        lo = orc.lin(hs_o, "class_embed")
        assert float((lg.double().cpu() - lo).abs().max()) <= 2e-3
        dg = model._mlp3(hs_g, model.bbox_embed)
        do = orc.mlp3(hs_o, "bbox_embed")
        bg = torch.cat([dg[..., :2] * ref_o[..., 2:].float().to(cuda) + ref_o[..., :2].float().to(cuda),
                        torch.exp(dg[..., 2:]) * ref_o[..., 2:].float().to(cuda)], -1)
        bo = torch.cat([do[..., :2] * ref_o[..., 2:] + ref_o[..., :2], torch.exp(do[..., 2:]) * ref_o[..., 2:]], -1)
        assert float((bg.double().cpu() - bo).abs().max()) <= 1e-3

        if np.array_equal(ig, io):
            boxes, logits = model(x.to(cuda))
            ob, ol = orc(x.double())
            assert float((logits.double().cpu() - ol).abs().max()) <= 2e-3
            assert float((boxes.double().cpu() - ob).abs().max()) <= 1e-3
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
