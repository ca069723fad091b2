"""The float64 oracle restatements agree with torch's independent CPU operators (a check of the oracle itself)."""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

import oracle.kernels as OK


def test_residual_layernorm_vs_torch():
    r = np.random.default_rng(0)
    h, o = r.standard_normal((64, 384)), r.standard_normal((64, 384))
    b, s, g, be = (r.standard_normal(384) for _ in range(4))
    ho, y = OK.residual_layernorm(h, o, b, s, g, be, 1e-6)
    th = torch.from_numpy(h) + (torch.from_numpy(o) + torch.from_numpy(b)) * torch.from_numpy(s)
    ty = F.layer_norm(th, (384,), torch.from_numpy(g), torch.from_numpy(be), 1e-6)
    assert np.abs(ho - th.numpy()).max() < 1e-12 and np.abs(y - ty.numpy()).max() < 1e-10


def test_linear_gelu_vs_torch():
    r = np.random.default_rng(1)
    x, w, b = r.standard_normal((50, 384)), 0.02 * r.standard_normal((384, 1536)), r.standard_normal(1536)
    ref = F.gelu(torch.from_numpy(x) @ torch.from_numpy(w) + torch.from_numpy(b), approximate="none")
    assert np.abs(OK.linear_gelu_f32(x, w, b) - ref.numpy()).max() < 1e-12


def test_deform_vs_grid_sample():
    """Per head and point, the oracle's sampling equals F.grid_sample(bilinear, zeros, align_corners=False) on
    grid 2*loc - 1 (ONNX GridSample semantics, fast_rfdetr/kernels.py:119-121)."""
    r = np.random.default_rng(2)
    b, nq, nh, hd, npts, gh, gw = 2, 30, 4, 8, 2, 10, 12
    value = r.standard_normal((b, gh * gw, 64))
    loc = r.uniform(-0.1, 1.1, (b, nq, nh, npts, 2))
    aw = r.uniform(0, 1, (b, nq, nh, npts))
    off = 16
    ours = OK.deform_attn(value, loc, aw, (gh, gw), nh, hd, off)
    v = torch.from_numpy(value[:, :, off:off + nh * hd]).reshape(b, gh, gw, nh, hd).permute(0, 3, 4, 1, 2)
    v = v.reshape(b * nh, hd, gh, gw)
    grid = torch.from_numpy(2 * loc - 1).permute(0, 2, 1, 3, 4).reshape(b * nh, nq, npts, 2)
    s = F.grid_sample(v, grid, mode="bilinear", padding_mode="zeros", align_corners=False)   # [b*nh, hd, nq, np]
    s = s.reshape(b, nh, hd, nq, npts).permute(0, 3, 1, 4, 2)                                # [b, nq, nh, np, hd]
    ref = (s * torch.from_numpy(aw)[..., None]).sum(3).reshape(b, nq, nh * hd)
    assert np.abs(ours - ref.numpy()).max() < 1e-10
