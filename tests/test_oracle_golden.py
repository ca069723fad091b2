"""Pins the CPU oracle and the native table generator to the reference (no GPU needed).

The fixtures in tests/golden/ were generated from the reference's own resize_tables.py (make_golden.py):
tables for 21 sizes under both policies, and sha256 digests of its resize_reference() output on the seeded
images of the reference test (tests/test_fast_rfdetr.py:40-43).
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import oracle.resize as OR
from kernelopt_b200 import resize_tables as RT

GOLD = Path(__file__).parent / "golden"
TABLES = np.load(GOLD / "resize_tables.npz")
DIGESTS = json.loads((GOLD / "resize_digests.json").read_text())["digests"]
SIZES = sorted({tuple(int(v) for v in k.split("_")[1].split("x")) for k in TABLES.files})


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def seeded(h, w):
    return np.random.default_rng(h * w).integers(0, 256, (h, w, 3), dtype=np.uint8)


@pytest.mark.parametrize("policy", ["reference", "opencv"])
@pytest.mark.parametrize("hw", SIZES)
def test_oracle_tables_match_reference(policy, hw):
    h, w = hw
    key = f"{policy}_{h}x{w}"
    mode, xt, yt = OR.tables(w, h, 640, 640, policy)
    assert mode == int(TABLES[key + "_mode"])
    assert np.array_equal(xt, TABLES[key + "_xtab"])
    assert np.array_equal(yt, TABLES[key + "_ytab"])


@pytest.mark.parametrize("policy", ["reference", "opencv"])
@pytest.mark.parametrize("hw", SIZES)
def test_native_tables_match_reference(policy, hw):
    h, w = hw
    key = f"{policy}_{h}x{w}"
    mode, xt, yt = RT.tables(w, h, 640, 640, policy)
    assert mode == int(TABLES[key + "_mode"])
    assert np.array_equal(xt, TABLES[key + "_xtab"])
    assert np.array_equal(yt, TABLES[key + "_ytab"])


@pytest.mark.parametrize("size", sorted(DIGESTS))
def test_oracle_resize_digests(size):
    h, w = (int(v) for v in size.split("x"))
    img = seeded(h, w)
    d = DIGESTS[size]
    assert sha(OR.resize(img, policy="reference")) == d["reference"]
    assert sha(OR.resize(img, policy="opencv")) == d["opencv"]


@pytest.mark.parametrize("size", sorted(DIGESTS))
def test_opencv_policy_is_cv2(size):
    """On a cv2 build without KleidiCV the opencv-policy tables are cv2.resize, and the LUT normalisation is
    Ballform's float32 preprocessing, bit for bit."""
    cv2 = pytest.importorskip("cv2")
    h, w = (int(v) for v in size.split("x"))
    img = seeded(h, w)
    resized = cv2.resize(img, (640, 640))
    assert sha(resized) == DIGESTS[size]["cv2"], "this machine's cv2 differs from the one the fixtures record"
    assert sha(OR.resize(img, policy="opencv")) == sha(resized)
    assert sha(OR.preprocess(img, policy="opencv")) == DIGESTS[size]["cv2_preprocess_hwc_f32"]


def test_lut_equals_float32_normalisation():
    v = np.arange(256, dtype=np.uint8)
    img = np.stack([v, v[::-1], np.roll(v, 7)], -1)[None]      # [1, 256, 3] BGR
    direct = OR.normalize(img)[0]                               # [256, 3] RGB
    lut = OR.lut()
    via_lut = np.stack([lut[c][img[0, :, 2 - c]] for c in range(3)], -1)
    assert np.array_equal(direct.view(np.uint32), via_lut.view(np.uint32))


def test_wide_outputs_cross_check():
    """Outputs wider than 2736 px exercise the KleidiCV coordinate resync; oracle and native must agree."""
    for sw, sh, dw, dh in [(9000, 1080, 3000, 500), (8000, 2000, 2900, 300)]:
        a = OR.tables(sw, sh, dw, dh)
        b = RT.tables(sw, sh, dw, dh)
        assert a[0] == b[0] == 0 and np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])


def test_tables_reject_bad_arguments():
    with pytest.raises(ValueError):
        RT.tables(1920, 1080, policy="nearest")
    with pytest.raises(ValueError):
        RT.tables(0, 1080)
