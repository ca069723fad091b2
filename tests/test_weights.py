"""Weight schema, safetensors round trip and load_weights dispatch (CPU)."""
from __future__ import annotations

import numpy as np
import pytest

from kernelopt_b200 import weights as W
from kernelopt_b200.detector import load_weights


def test_random_weights_schema_and_determinism():
    a, b = W.random_weights(3), W.random_weights(3)
    assert a.keys() == b.keys()
    assert all(np.array_equal(a[k], b[k]) for k in a)
    assert a[W.BB + "embeddings.patch_embeddings.projection.weight"].shape == (384, 16, 16, 3)
    assert a[W.LAYER.format(11) + "mlp.fc1.weight"].shape == (384, 1536)
    assert a[W.PROJ + "0.m.2.cv2.conv.weight"].shape == (128, 3, 3, 128)
    assert a["proposals"].shape == (1600, 4) and a["proposal_valid"].min() == 1.0
    assert float(np.asarray(a["_eps." + W.LAYER.format(0) + "norm1.weight"]).reshape(())) == pytest.approx(1e-6)
    w = a[W.LAYER.format(0) + "mlp.fc2.weight"]
    assert np.abs(w).max() <= 0.04 + 1e-7 and 0.015 < w.std() < 0.02


def test_safetensors_round_trip_and_load_weights(tmp_path):
    w = W.random_weights(1)
    path = tmp_path / "mlx-cache" / "abc" / "weights.safetensors"
    W.save(w, path)
    back = load_weights(path)
    assert back.keys() == w.keys() and all(np.array_equal(back[k], w[k]) for k in w)
    assert load_weights("random:1").keys() == w.keys()


def test_load_weights_onnx_uses_reference_cache(tmp_path):
    onnx = tmp_path / "model.onnx"
    onnx.write_bytes(b"not really onnx")
    with pytest.raises(RuntimeError):
        load_weights(onnx)
    cache = tmp_path / "cache"
    W.save(W.random_weights(2), cache / "weights.safetensors")
    assert "query_feat" in load_weights(onnx, cache_dir=cache)
    with pytest.raises(ValueError):
        load_weights(tmp_path / "model.pt")
