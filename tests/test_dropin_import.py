"""The reference's import path works unchanged: `fast_rfdetr` and its kernels / detector / resize_tables modules
expose the B200 objects (fast_rfdetr/__init__.py:2-4, fast_rfdetr/model.py:9 of the reference)."""
from __future__ import annotations

import numpy as np
import pytest

import kernelopt_b200.detector as KD
import kernelopt_b200.kernels as KK
import kernelopt_b200.resize_tables as KR


def test_reference_imports_resolve_to_the_b200_objects():
    from fast_rfdetr import FastBasketballDetector, load_weights
    from fast_rfdetr.kernels import deform_attn, linear_gelu_f32, preprocess_gpu, residual_layernorm
    from fast_rfdetr.resize_tables import tables, uses_kleidicv

    assert FastBasketballDetector is KD.FastBasketballDetector and load_weights is KD.load_weights
    assert (residual_layernorm, preprocess_gpu, deform_attn, linear_gelu_f32) == (
        KK.residual_layernorm, KK.preprocess_gpu, KK.deform_attn, KK.linear_gelu_f32)
    assert tables is KR.tables and uses_kleidicv is KR.uses_kleidicv
    import fast_rfdetr
    assert set(fast_rfdetr.__all__) == {"FastBasketballDetector", "load_weights"}
    with pytest.raises(AttributeError):
        fast_rfdetr.not_a_name  # noqa: B018


def test_reference_table_api_through_the_import_path():
    from fast_rfdetr.resize_tables import tables, uses_kleidicv

    mode, xt, yt = tables(1920, 1080, 640, 640)
    assert mode == 0 and uses_kleidicv(1920, 1080, 640, 640)
    assert xt.shape == (640 * 3, 4) and yt.shape == (640, 4) and xt.dtype == np.int32
    assert tables(960, 540)[0] == 1 and not uses_kleidicv(960, 540, 640, 640)


def test_reference_model_and_weights_modules():
    from fast_rfdetr.model import RFDETR, TAPS
    from fast_rfdetr.weights import proposals

    import kernelopt_b200.model as KM
    assert RFDETR is KM.RFDETR and TAPS == (2, 5, 8, 11)
    assert proposals()["proposals"].shape == (1600, 4)


@pytest.mark.gpu
def test_kernel_through_the_reference_import_path(cuda):
    """residual_layernorm called exactly as the reference's model calls it (model.py:122), on CUDA tensors."""
    import torch

    import oracle.kernels as OK
    from fast_rfdetr.kernels import residual_layernorm

    r = np.random.default_rng(5)
    h, o = (r.standard_normal((1604, 384)).astype(np.float32) for _ in range(2))
    bias, gamma, beta = (0.1 * r.standard_normal(384)).astype(np.float32), \
        (1 + 0.1 * r.standard_normal(384)).astype(np.float32), (0.1 * r.standard_normal(384)).astype(np.float32)
    scale = (1 + 0.1 * r.standard_normal(384)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    h_out, y = residual_layernorm(t(h), t(o), t(bias), t(scale), t(gamma), t(beta), 1e-6)
    rh, ry = OK.residual_layernorm(h, o, bias, scale, gamma, beta, 1e-6)
    for g, ref in ((h_out, rh), (y, ry)):
        g = g.double().cpu().numpy()
        assert np.abs(g - ref).max() <= 1e-5 * np.abs(ref).max()
