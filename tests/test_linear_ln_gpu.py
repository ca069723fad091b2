"""GEMM + residual + LayerNorm in one kernel (ko_linear_residual_ln_f32_packed) against the float64 oracle.

Cases: the backbone's out-projection (K 384) and fc2 (K 1536, the correction accumulator) at N 384, where a row
spans a cluster of two CTAs; the decoder's N 256 sites (K 256 and 2048); the projector's GEMM + LayerNorm + SiLU
without a residual (N 128 / 256); ragged row counts, in-place residual, determinism and the rejected widths.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.kernels as OK
from kernelopt_b200 import _lib
from kernelopt_b200 import kernels as K

pytestmark = pytest.mark.gpu

REL = 1e-5


def assert_close(gpu, ref, rel=REL, what=""):
    gpu = gpu.detach().cpu().double().numpy()
    ref = np.asarray(ref, np.float64)
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    assert np.isfinite(gpu).all(), f"{what}: non-finite output"
    err = np.abs(gpu - ref).max()
    scale = np.abs(ref).max()
    assert err <= rel * scale, f"{what}: normwise error {err / scale:.3e} > {rel}"


def make(m, k, n, seed, resid=True, scale=True, bias=True):
    r = np.random.default_rng(seed)
    d = dict(
        x=r.standard_normal((m, k)).astype(np.float32),
        w=(r.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32),
        bias=(0.1 * r.standard_normal(n)).astype(np.float32) if bias else None,
        scale=(1.0 + 0.1 * r.standard_normal(n)).astype(np.float32) if scale else None,
        resid=r.standard_normal((m, n)).astype(np.float32) if resid else None,
        gamma=(1.0 + 0.1 * r.standard_normal(n)).astype(np.float32),
        beta=(0.1 * r.standard_normal(n)).astype(np.float32),
    )
    return d


def run(cuda, d, eps=1e-6, act=None, in_place=False, write_h=True):
    t = lambda a: None if a is None else torch.from_numpy(a).to(cuda)  # noqa: E731
    pw = K.pack_weight(t(d["w"]), t(d["bias"]))
    resid = t(d["resid"])
    h_out, y = K.linear_residual_layernorm(t(d["x"]), pw, t(d["gamma"]), t(d["beta"]), eps, resid=resid,
                                           scale=t(d["scale"]), act=act, h_out=resid if in_place else None,
                                           write_h=write_h)
    torch.cuda.synchronize()
    K.check_device_status()
    return h_out, y


@pytest.mark.parametrize("m,k,n", [(3208, 384, 384), (3208, 1536, 384), (102656 // 8, 384, 384), (1, 384, 384),
                                   (129, 1536, 384), (2400, 256, 256), (2400, 2048, 256), (1000, 320, 192),
                                   (777, 512, 512), (130, 640, 128), (40000, 384, 256)])
def test_linear_residual_ln(cuda, m, k, n):
    # N = 256 runs as a cluster of two 128-wide CTAs below two row blocks per SM (2400 rows) and as one
    # 256-wide CTA above (40000 rows).
    d = make(m, k, n, m + k + n)
    h_out, y = run(cuda, d)
    rh, ry = OK.linear_residual_layernorm(d["x"], d["w"], d["bias"], d["scale"], d["resid"], d["gamma"], d["beta"],
                                          1e-6)
    assert_close(h_out, rh, what=f"h_out {m}x{k}x{n}")
    assert_close(y, ry, what=f"y {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n", [(1600, 1152, 128), (1600, 768, 256), (1600, 2304, 256), (1600, 256, 128),
                                   (3000, 384, 256), (2000, 384, 384)])
def test_linear_ln_silu_no_residual(cuda, m, k, n):
    """The projector's conv-as-GEMM -> channel LayerNorm -> SiLU (no residual, no scale, LN eps 1e-6); K <= 512
    also runs the epilogue with two staging tiles per warp without any residual load or v store."""
    d = make(m, k, n, 7 * n, resid=False, scale=False)
    h_out, y = run(cuda, d, act="silu", write_h=False)
    assert h_out is None
    _, ry = OK.linear_residual_layernorm(d["x"], d["w"], d["bias"], None, None, d["gamma"], d["beta"], 1e-6, "silu")
    assert_close(y, ry, what=f"silu {m}x{k}x{n}")


def test_in_place_residual_and_determinism(cuda):
    d = make(4100, 1536, 384, 5)
    rh, ry = OK.linear_residual_layernorm(d["x"], d["w"], d["bias"], d["scale"], d["resid"], d["gamma"], d["beta"],
                                          1e-6)
    h1, y1 = run(cuda, d, in_place=True)
    h2, y2 = run(cuda, d)
    assert_close(h1, rh, what="in place h")
    assert_close(y1, ry, what="in place y")
    assert torch.equal(h1, h2) and torch.equal(y1, y2), "results differ between runs / in place"


def test_matches_unfused_pair(cuda):
    """Same values as the GEMM followed by the stand-alone residual + LayerNorm kernel (both fp32-grade)."""
    d = make(3208, 384, 384, 11)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    h, y = run(cuda, d)
    o = K.linear(t(d["x"]), K.pack_weight(t(d["w"])))
    h2, y2 = K.residual_layernorm(t(d["resid"]), o, t(d["bias"]), t(d["scale"]), t(d["gamma"]), t(d["beta"]), 1e-6)
    torch.cuda.synchronize()
    assert (h - h2).abs().max().item() <= 1e-5 * h2.abs().max().item()
    assert (y - y2).abs().max().item() <= 1e-5 * y2.abs().max().item()


def test_rejects_unsupported_width(cuda):
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    d = make(64, 64, 320, 3)
    pw = K.pack_weight(t(d["w"]))
    with pytest.raises(ValueError):
        K.linear_residual_layernorm(t(d["x"]), pw, t(d["gamma"]), t(d["beta"]), 1e-6)
    y = torch.empty((64, 320), device=cuda)
    with pytest.raises(_lib.KernelError):
        _lib.call("ko_linear_residual_ln_f32_packed", t(d["x"]).data_ptr(), pw.packed.data_ptr(), None, None, None,
                  t(d["gamma"]).data_ptr(), t(d["beta"]).data_ptr(), 1e-6, 64, 64, 320, 0, None, y.data_ptr(), 0,
                  None, torch.cuda.current_stream().cuda_stream)


def test_empty_rows(cuda):
    d = make(1, 384, 384, 1)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    pw = K.pack_weight(t(d["w"]))
    x = torch.empty((0, 384), device=cuda)
    h, y = K.linear_residual_layernorm(x, pw, t(d["gamma"]), t(d["beta"]), 1e-6)
    assert h.shape == (0, 384) and y.shape == (0, 384)


def im2col3x3_np(x):
    b, h, w, c = x.shape
    xp = np.pad(x, ((0, 0), (1, 1), (1, 1), (0, 0)))
    return np.concatenate([xp[:, dy:dy + h, dx:dx + w] for dy in range(3) for dx in range(3)], -1).reshape(
        b * h * w, 9 * c)


@pytest.mark.parametrize("b,h,w,c,n", [(2, 40, 40, 128, 128), (1, 7, 5, 16, 128), (3, 40, 40, 128, 256),
                                       (1, 1, 1, 32, 128), (2, 9, 13, 48, 384)])
def test_conv3x3_ln_silu(cuda, b, h, w, c, n):
    """Implicit-GEMM 3x3 convolution + LayerNorm + SiLU against im2col + GEMM + LN + SiLU in float64."""
    r = np.random.default_rng(b * 1000 + h * 10 + c)
    x = r.standard_normal((b, h, w, c)).astype(np.float32)
    wt = (r.standard_normal((9 * c, n)) / np.sqrt(9 * c)).astype(np.float32)
    bias = (0.1 * r.standard_normal(n)).astype(np.float32)
    gamma = (1.0 + 0.1 * r.standard_normal(n)).astype(np.float32)
    beta = (0.1 * r.standard_normal(n)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    pw = K.pack_weight(t(wt), t(bias))
    y = K.conv3x3_layernorm(t(x), pw, t(gamma), t(beta), 1e-6, act="silu")
    torch.cuda.synchronize()
    K.check_device_status()
    _, ry = OK.linear_residual_layernorm(im2col3x3_np(x), wt, bias, None, None, gamma, beta, 1e-6, "silu")
    assert_close(y, ry, what=f"conv {b}x{h}x{w}x{c}->{n}")
    # the same values as the explicit im2col path
    _, y2 = K.linear_residual_layernorm(K.im2col3x3(t(x)), pw, t(gamma), t(beta), 1e-6, act="silu", write_h=False)
    torch.cuda.synchronize()
    assert (y - y2).abs().max().item() <= 1e-5 * y2.abs().max().item()


def test_conv3x3_rejects_bad_channels(cuda):
    x = torch.zeros((1, 4, 4, 20), device=cuda)
    pw = K.pack_weight(torch.zeros((180, 128), device=cuda))
    with pytest.raises(ValueError):
        K.conv3x3_layernorm(x, pw, torch.ones(128, device=cuda), torch.zeros(128, device=cuda), 1e-6)
