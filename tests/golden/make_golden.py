"""Generates the golden fixtures that pin the preprocessing oracle to the reference's own code.

Run in a container where the reference checkout is available (it is NOT needed at test time):

    python tests/golden/make_golden.py /path/to/kernelopt-reference

It imports the reference's pure-numpy table model (fast_rfdetr/resize_tables.py — the only part of the
reference that runs without MLX and Apple hardware) straight from its file and records:

  resize_tables.npz   mode / xtab / ytab for every size below, under the reference's own policy and with its
                      KleidiCV selection switched off (the table set a cv2 build without KleidiCV uses).
  resize_digests.json sha256 of the reference's resize_reference() output on the seeded noise images of the
                      reference test (default_rng(h*w), tests/test_fast_rfdetr.py:40-43) under both policies,
                      the sha256 of cv2.resize on this machine, and the sha256 of Ballform's float32
                      preprocessing (tests/test_fast_rfdetr.py:25-27) for the same images.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path
from unittest import mock

import numpy as np

HERE = Path(__file__).parent

# Sizes of the reference test (tests/test_fast_rfdetr.py:40), its 20-size sweep (rfdetr/check_resize.py:11-13)
# and the benchmark frame sizes (1920x1080, 1280x720, 960x540). (h, w).
SIZES = sorted({(1080, 1920), (1080, 1152), (720, 1280), (500, 333), (2160, 3840), (641, 1279), (480, 640),
                (640, 640), (300, 1000), (700, 700), (1000, 300), (1079, 1919), (1080, 1100), (650, 1900),
                (1440, 2560), (1200, 1600), (900, 1000), (1081, 1921), (720, 960), (645, 645), (540, 960)})
DIGEST_SIZES = [(1080, 1920), (1080, 1152), (720, 1280), (500, 333), (2160, 3840), (641, 1279), (540, 960)]
MEAN = np.asarray([.485, .456, .406], dtype=np.float32)
STD = np.asarray([.229, .224, .225], dtype=np.float32)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref_root: str) -> None:
    spec = importlib.util.spec_from_file_location("ref_resize_tables",
                                                  Path(ref_root) / "fast_rfdetr" / "resize_tables.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    import cv2

    arrays = {}
    for policy in ("reference", "opencv"):
        patch = mock.patch.object(ref, "uses_kleidicv", lambda *a: False) if policy == "opencv" else mock.MagicMock()
        with patch:
            ref.tables.cache_clear()
            for h, w in SIZES:
                mode, xt, yt = ref.tables(w, h, 640, 640)
                key = f"{policy}_{h}x{w}"
                arrays[key + "_mode"] = np.asarray(mode, np.int32)
                arrays[key + "_xtab"] = xt
                arrays[key + "_ytab"] = yt
    ref.tables.cache_clear()
    np.savez_compressed(HERE / "resize_tables.npz", **arrays)

    digests = {}
    for h, w in DIGEST_SIZES:
        img = np.random.default_rng(h * w).integers(0, 256, (h, w, 3), dtype=np.uint8)
        entry = {"reference": sha(ref.resize_reference(img))}
        with mock.patch.object(ref, "uses_kleidicv", lambda *a: False):
            ref.tables.cache_clear()
            entry["opencv"] = sha(ref.resize_reference(img))
        ref.tables.cache_clear()
        resized = cv2.resize(img, (640, 640))
        entry["cv2"] = sha(resized)
        rgb = cv2.cvtColor(resized, cv2.COLOR_BGR2RGB).astype(np.float32) / 255.
        entry["cv2_preprocess_hwc_f32"] = sha(((rgb - MEAN) / STD).astype(np.float32))
        digests[f"{h}x{w}"] = entry
    meta = {"cv2_version": cv2.__version__, "numpy_version": np.__version__, "images": "default_rng(h*w) uniform u8",
            "digests": digests}
    (HERE / "resize_digests.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
