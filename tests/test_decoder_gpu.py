"""The decoder and head kernels against float64 references: the sine embedding, the narrow fp32 linear layer and
the fused box head (fast_rfdetr/model.py:188-194, :179-180, :269-272), the GEMM with an added per-element term
(the decoder's (tgt + qpos) @ W = tgt @ W + qpos @ W, model.py:251, :256), and the LayerNorm GEMMs writing into /
reading from channel slices of a wider buffer (the projector's in-place concatenation, model.py:161-162)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle.kernels as OK
from kernelopt_b200 import kernels as K
from kernelopt_b200.weights import dim_t

pytestmark = pytest.mark.gpu
REL = 1e-5


def close(g, ref, rel=REL, what=""):
    g = g.detach().double().cpu().numpy()
    ref = np.asarray(ref, np.float64)
    err = np.abs(g - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err <= rel, f"{what}: relative error {err:.2e}"


def t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("rows", [1, 300, 19200])
def test_sine_embed(cuda, rows):
    r = np.random.default_rng(rows)
    ref = r.uniform(0, 1, (rows, 4)).astype(np.float32)
    dt = dim_t()
    g = K.sine_embed(t(ref, cuda), t(dt, cuda))
    outs = []
    for c in (1, 0, 2, 3):
        v = (ref[:, c].astype(np.float64) * 2 * math.pi)[:, None] / dt.astype(np.float64)
        outs.append(np.stack([np.sin(v[:, 0::2]), np.cos(v[:, 1::2])], -1).reshape(rows, 128))
    want = np.concatenate(outs, -1)
    assert float(np.abs(g.double().cpu().numpy() - want).max()) <= 2e-6   # sin / cos of fp32 arguments


@pytest.mark.parametrize("m,k,n,act", [(19200, 256, 11, None), (102400, 256, 11, None), (300, 256, 4, None),
                                       (7, 256, 11, "relu"), (1, 100, 32, None), (333, 48, 17, "relu"),
                                       (5, 256, 16, None), (33, 256, 1, "relu"), (1000, 256, 5, None),
                                       (64, 256, 20, None)])
def test_linear_small(cuda, m, k, n, act):
    r = np.random.default_rng(m + k + n)
    x = r.standard_normal((m, k)).astype(np.float32)
    w = (0.05 * r.standard_normal((k, n))).astype(np.float32)
    b = (0.1 * r.standard_normal(n)).astype(np.float32)
    g = K.linear_small(t(x, cuda), t(w, cuda), t(b, cuda), act)
    close(g, OK.linear(x, w, b, act), what=f"linear_small {m}x{k}x{n}")


def test_box_head(cuda):
    r = np.random.default_rng(4)
    x = r.standard_normal((2, 300, 256)).astype(np.float32)
    w = (0.02 * r.standard_normal((256, 4))).astype(np.float32)
    b = (0.01 * r.standard_normal(4)).astype(np.float32)
    ref = np.concatenate([r.uniform(0.1, 0.9, (2, 300, 2)), r.uniform(0.01, 0.2, (2, 300, 2))], -1).astype(np.float32)
    g = K.box_head(t(x, cuda), t(w, cuda), t(b, cuda), t(ref, cuda))
    d = x.astype(np.float64) @ w + b
    r64 = ref.astype(np.float64)
    want = np.concatenate([d[..., :2] * r64[..., 2:] + r64[..., :2], np.exp(d[..., 2:]) * r64[..., 2:]], -1)
    close(g, want, what="box head")


@pytest.mark.parametrize("m,k,n,add_cols,ld", [(600, 256, 768, 512, 2432), (19200, 256, 96, 96, 2432),
                                               (130, 64, 128, 64, 64)])
def test_linear_add(cuda, m, k, n, add_cols, ld):
    r = np.random.default_rng(m + n)
    x = r.standard_normal((m, k)).astype(np.float32)
    w = (0.05 * r.standard_normal((k, n))).astype(np.float32)
    b = (0.1 * r.standard_normal(n)).astype(np.float32)
    wide = r.standard_normal((m, ld)).astype(np.float32)
    off = (ld - add_cols) // 4 * 4
    addend = t(wide, cuda)[:, off:off + add_cols]
    g = K.linear_add(t(x, cuda), K.pack_weight(t(w, cuda), t(b, cuda)), addend)
    want = x.astype(np.float64) @ w + b
    want[:, :add_cols] += wide[:, off:off + add_cols]
    torch.cuda.synchronize()
    K.check_device_status()
    close(g, want, what="linear + addend")
    with pytest.raises(ValueError):
        K.linear_add(t(x, cuda), K.pack_weight(t(w, cuda)), addend[:-1])


def test_layernorm_gemms_on_channel_slices(cuda):
    """cv1-style 1x1 conv writing channels [0, 256) of a 640-wide NHWC buffer, and a 3x3 conv reading channels
    [128, 256) of it and writing channels [256, 384): bit-identical to the same kernels on dense tensors, and the
    channels they do not own are left untouched."""
    r = np.random.default_rng(12)
    b, hw, c_in = 2, 40, 1536
    x = t(r.standard_normal((b, hw, hw, c_in)).astype(np.float32), cuda)
    w1 = t((r.standard_normal((c_in, 256)) / math.sqrt(c_in)).astype(np.float32), cuda)
    w3 = t((r.standard_normal((9 * 128, 128)) / math.sqrt(9 * 128)).astype(np.float32), cuda)
    g1, b1 = t((1 + 0.1 * r.standard_normal(256)).astype(np.float32), cuda), t(
        (0.1 * r.standard_normal(256)).astype(np.float32), cuda)
    g3, b3 = g1[:128].contiguous(), b1[:128].contiguous()
    pw1, pw3 = K.pack_weight(w1), K.pack_weight(w3)
    cat = torch.full((b, hw, hw, 640), 7.0, device=cuda)
    K.linear_residual_layernorm(x.reshape(-1, c_in), pw1, g1, b1, 1e-6, act="silu", y=cat[..., :256], write_h=False)
    K.conv3x3_layernorm(cat[..., 128:256], pw3, g3, b3, 1e-6, "silu", out=cat[..., 256:384])
    _, dense1 = K.linear_residual_layernorm(x.reshape(-1, c_in), pw1, g1, b1, 1e-6, act="silu", write_h=False)
    dense1 = dense1.reshape(b, hw, hw, 256)
    dense3 = K.conv3x3_layernorm(dense1[..., 128:].contiguous(), pw3, g3, b3, 1e-6, "silu").reshape(b, hw, hw, 128)
    torch.cuda.synchronize()
    K.check_device_status()
    assert torch.equal(cat[..., :256], dense1)
    assert torch.equal(cat[..., 256:384], dense3)
    assert bool((cat[..., 384:] == 7.0).all())
