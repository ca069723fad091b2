"""Parity of the four CUDA kernels with the CPU oracle, through the C ABI (libkernelopt.so via ctypes).

Tolerances:
  preprocessing  bit-exact (float32 bit patterns compared as uint32)
  fp32 kernels   relative error <= 1e-5 in the max norm against the float64 oracle:
                 max|gpu - ref| <= 1e-5 * max|ref| over the output tensor. (A per-element relative bound is
                 meaningless where outputs cross zero; fp32 rounding of the sampling coordinates alone moves
                 deform outputs by ~1e-6 of the map's scale, in the reference kernel as in this one.)
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle.kernels as OK
import oracle.resize as OR
from kernelopt_b200 import kernels as K
from kernelopt_b200 import resize_tables as RT

pytestmark = pytest.mark.gpu

REL = 1e-5


def assert_close(gpu, ref, rel=REL, what=""):
    gpu = gpu.detach().cpu().double().numpy() if isinstance(gpu, torch.Tensor) else np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    err = np.abs(gpu - ref)
    scale = np.abs(ref).max()
    assert np.isfinite(gpu).all(), f"{what}: non-finite output"
    assert err.max() <= rel * scale, f"{what}: normwise error {err.max() / scale:.3e} > {rel}"


def gpu_lut(dev):
    return torch.from_numpy(OR.lut()).to(dev)


def frame(h, w, seed, kind="noise"):
    if kind == "noise":
        return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)
    y, x = np.mgrid[0:h, 0:w]
    return np.stack([(x * 255 // max(w - 1, 1)), (y * 255 // max(h - 1, 1)), ((x + y) * 255 // max(h + w - 2, 1))],
                    -1).astype(np.uint8)


# ---------------------------------------------------------------- preprocessing
@pytest.mark.parametrize("policy", ["reference", "opencv"])
@pytest.mark.parametrize("hw", [(1080, 1920), (720, 1280), (540, 960), (1080, 1152), (500, 333), (641, 1279),
                                (2160, 3840), (480, 640), (1000, 300)])
def test_preprocess_bit_exact(cuda, policy, hw):
    h, w = hw
    lut = gpu_lut(cuda)
    for kind in ("noise", "gradient"):
        img = frame(h, w, h * w, kind)
        mode, xt, yt = RT.tables(w, h, policy=policy)
        g = K.preprocess_gpu(torch.from_numpy(img).to(cuda), torch.from_numpy(np.array(xt)).to(cuda),
                             torch.from_numpy(np.array(yt)).to(cuda), lut, mode)
        ref = OR.preprocess(img, policy=policy)
        assert np.array_equal(g.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (policy, hw, kind)


def test_preprocess_matches_cv2_opencv_policy(cuda):
    cv2 = pytest.importorskip("cv2")
    lut = gpu_lut(cuda)
    for h, w in [(1080, 1920), (720, 1280), (540, 960)]:
        img = frame(h, w, 7 + h)
        mode, xt, yt = RT.tables(w, h, policy="opencv")
        g = K.preprocess_gpu(torch.from_numpy(img).to(cuda), torch.from_numpy(np.array(xt)).to(cuda),
                             torch.from_numpy(np.array(yt)).to(cuda), lut, mode, layout="chw")
        rgb = cv2.cvtColor(cv2.resize(img, (640, 640)), cv2.COLOR_BGR2RGB).astype(np.float32) / 255.
        ref = np.ascontiguousarray(((rgb - OR.MEAN) / OR.STD).transpose(2, 0, 1))
        assert np.array_equal(g.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("layout", ["hwc", "chw", "patch16"])
def test_preprocess_batch_mixed_sizes(cuda, layout):
    lut = gpu_lut(cuda)
    sizes = [(1080, 1920), (720, 1280), (540, 960)]
    imgs = [frame(h, w, 100 + i) for i, (h, w) in enumerate(sizes)]
    items, refs = [], []
    for img in imgs:
        h, w, _ = img.shape
        mode, xt, yt = RT.tables(w, h)
        items.append((torch.from_numpy(img).to(cuda), torch.from_numpy(np.array(xt)).to(cuda),
                      torch.from_numpy(np.array(yt)).to(cuda), mode))
        refs.append(OR.preprocess(img, layout=layout))
    out = K.preprocess_batch(items, lut, layout=layout)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), np.stack(refs).view(np.uint32))


def test_preprocess_many_frames_use_row_bands(cuda):
    """16 frames of mixed sizes in one launch: the band kernel gives each CTA several output rows."""
    lut = gpu_lut(cuda)
    sizes = [(1080, 1920), (720, 1280), (540, 960), (641, 1279)]
    items, refs = [], []
    for i in range(16):
        h, w = sizes[i % 4]
        img = frame(h, w, 200 + i, "noise" if i % 2 == 0 else "gradient")
        mode, xt, yt = RT.tables(w, h)
        items.append((torch.from_numpy(img).to(cuda), torch.from_numpy(np.array(xt)).to(cuda),
                      torch.from_numpy(np.array(yt)).to(cuda), mode))
        refs.append(OR.preprocess(img, layout="patch16"))
    out = K.preprocess_batch(items, lut, layout="patch16")
    assert np.array_equal(out.cpu().numpy().view(np.uint32), np.stack(refs).view(np.uint32))


@pytest.mark.parametrize("policy", ["reference", "opencv"])
@pytest.mark.parametrize("layout", ["hwc", "patch16"])
@pytest.mark.parametrize("n_frames", [10, 24])
def test_preprocess_many_aligned_frames(cuda, policy, layout, n_frames):
    """Frames whose rows are whole 16-byte chunks (the segment kernel; 10 frames take 8-row bands, 24 take 16-row
    bands): each warp takes several tasks, crosses images of different sizes and table modes, and runs both the
    left-tap and the four-tap arithmetic."""
    lut = gpu_lut(cuda)
    sizes = [(1080, 1920), (720, 1280), (540, 960), (1080, 1152)]
    items, refs = [], []
    for i in range(n_frames):
        h, w = sizes[i % 4]
        img = frame(h, w, 300 + i, "noise" if i % 3 else "gradient")
        mode, xt, yt = RT.tables(w, h, policy=policy)
        items.append((torch.from_numpy(img).to(cuda), torch.from_numpy(np.array(xt)).to(cuda),
                      torch.from_numpy(np.array(yt)).to(cuda), mode))
        refs.append(OR.preprocess(img, policy=policy, layout=layout))
    out = K.preprocess_batch(items, lut, layout=layout)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), np.stack(refs).view(np.uint32))


def test_preprocess_benchmark_batch(cuda):
    """The benchmark's own case: 64 noise frames of 1920x1080 with OpenCV tables into PATCH16 (the segment
    kernel's left-tap path, 16-row bands, several tasks per warp), bit-exact against the oracle."""
    lut = gpu_lut(cuda)
    mode, xt, yt = RT.tables(1920, 1080, policy="opencv")
    xt_d, yt_d = torch.from_numpy(np.array(xt)).to(cuda), torch.from_numpy(np.array(yt)).to(cuda)
    rng = np.random.default_rng(64)
    imgs = [rng.integers(0, 256, (1080, 1920, 3), dtype=np.uint8) for _ in range(64)]
    out = K.preprocess_batch([(torch.from_numpy(im).to(cuda), xt_d, yt_d, mode) for im in imgs], lut,
                             layout="patch16").cpu().numpy()
    for i in range(0, 64, 7):  # every seventh frame: spans images at every position in the warps' task order
        ref = OR.preprocess(imgs[i], policy="opencv", layout="patch16")
        assert np.array_equal(out[i].view(np.uint32), ref.view(np.uint32)), i


@pytest.mark.parametrize("hw,dst,policy", [((1080, 1920), 96, "opencv"), ((500, 333), 160, "reference"),
                                           ((1080, 1920), 1024, "reference"), ((1080, 1920), 1024, "opencv"),
                                           ((500, 333), 1024, "reference")])
def test_preprocess_other_output_sizes(cuda, hw, dst, policy):
    """Outputs narrower than 342 (one item per thread), and wider than 682 (the one-row-per-CTA kernel)."""
    h, w = hw
    lut = gpu_lut(cuda)
    img = frame(h, w, dst + h)
    mode, xt, yt = RT.tables(w, h, dst, dst, policy=policy)
    for layout in ("hwc", "patch16"):
        g = K.preprocess_gpu(torch.from_numpy(img).to(cuda), torch.from_numpy(np.array(xt)).to(cuda),
                             torch.from_numpy(np.array(yt)).to(cuda), lut, mode, dst=dst, layout=layout)
        ref = OR.preprocess(img, dst=dst, policy=policy, layout=layout)
        assert np.array_equal(g.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (hw, dst, policy, layout)


def test_preprocess_rejects_bad_input(cuda):
    lut = gpu_lut(cuda)
    mode, xt, yt = RT.tables(1920, 1080)
    img = torch.zeros((1080, 1920, 3), dtype=torch.float32, device=cuda)
    with pytest.raises(ValueError):
        K.preprocess_gpu(img, torch.from_numpy(np.array(xt)).to(cuda), torch.from_numpy(np.array(yt)).to(cuda),
                         lut, mode)
    with pytest.raises(ValueError):
        K.preprocess_gpu(img.to(torch.uint8), torch.from_numpy(np.array(xt)).to(cuda),
                         torch.from_numpy(np.array(yt)).to(cuda), lut, mode, dst=320)


# ---------------------------------------------------------------- residual + LayerNorm
@pytest.mark.parametrize("batch", [1, 3, 64])
def test_residual_layernorm(cuda, batch):
    r = np.random.default_rng(batch)
    rows, c = batch * 1600, 384
    h = r.standard_normal((rows, c)).astype(np.float32)
    o = r.standard_normal((rows, c)).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    beta = (0.1 * r.standard_normal(c)).astype(np.float32)
    bias = (0.1 * r.standard_normal(c)).astype(np.float32)
    scale = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    ho, y = K.residual_layernorm(t(h), t(o), t(bias), t(scale), t(gamma), t(beta), 1e-6)
    rho, ry = OK.residual_layernorm(h, o, bias, scale, gamma, beta, 1e-6)
    assert_close(ho, rho, what="h_out")
    assert_close(y, ry, what="y")
    ho, y = K.residual_layernorm(t(h), t(o), None, None, t(gamma), t(beta), 1e-6)
    rho, ry = OK.residual_layernorm(h, o, None, None, gamma, beta, 1e-6)
    assert_close(ho, rho, what="h_out (no bias/scale)")
    assert_close(y, ry, what="y (no bias/scale)")


@pytest.mark.parametrize("c", [256, 128, 4, 1024])
def test_residual_layernorm_widths(cuda, c):
    r = np.random.default_rng(c)
    h = r.standard_normal((37, c)).astype(np.float32)
    o = r.standard_normal((37, c)).astype(np.float32)
    g = r.standard_normal(c).astype(np.float32)
    b = r.standard_normal(c).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    ho, y = K.residual_layernorm(t(h), t(o), t(b), t(g), t(g), t(b), 1e-5)
    rho, ry = OK.residual_layernorm(h, o, b, g, g, b, 1e-5)
    assert_close(ho, rho)
    assert_close(y, ry)


@pytest.mark.parametrize("c", [128, 256, 384])
@pytest.mark.parametrize("act", [None, "silu"])
def test_layernorm_plain_and_silu(cuda, c, act):
    """ko_layernorm: the residual kernel without the residual, optionally with SiLU on its output."""
    r = np.random.default_rng(c + (act is not None))
    x = (3 * r.standard_normal((1000, c)) + 0.5).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    b = (0.1 * r.standard_normal(c)).astype(np.float32)
    _, ref = OK.residual_layernorm(x, np.zeros_like(x), None, None, g, b, 1e-5)
    if act == "silu":
        ref = ref / (1 + np.exp(-ref))
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    assert_close(K.layernorm(t(x), t(g), t(b), 1e-5, act), ref, what=f"layernorm c={c} act={act}")


@pytest.mark.parametrize("b,grid,win,c", [(2, (40, 40), 20, 384), (3, (8, 12), 4, 64), (1, (6, 6), 3, 1024),
                                          (2, (5, 10), 5, 132)])
def test_window_merge_layernorm(cuda, b, grid, win, c):
    """ko_window_merge_ln: window-ordered tokens (class token first) -> NHWC channel slice of a wider buffer,
    LayerNorm'd (1e-5 of the float64 LayerNorm) or copied (bit-exact); the channels around the slice untouched."""
    gh, gw = grid
    nwin = (gh // win) * (gw // win)
    r = np.random.default_rng(c + win)
    h = (2 * r.standard_normal((b * nwin, 1 + win * win, c)) + 0.3).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    bt = (0.1 * r.standard_normal(c)).astype(np.float32)
    _, ln = OK.residual_layernorm(h.reshape(-1, c), np.zeros((h.shape[0] * h.shape[1], c), np.float32), None, None,
                                  g, bt, 1e-6)
    merge = lambda a: a.reshape(b, gh // win, gw // win, 1 + win * win, c)[:, :, :, 1:].reshape(  # noqa: E731
        b, gh // win, gw // win, win, win, c).transpose(0, 1, 3, 2, 4, 5).reshape(b, gh, gw, c)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    out = torch.full((b, gh, gw, 3 * c + 8), 7.0, device=cuda)
    K.window_merge_layernorm(t(h), grid, win, out, 4, t(g), t(bt), 1e-6)
    K.window_merge_layernorm(t(h), grid, win, out, 4 + 2 * c, normalize=False)
    torch.cuda.synchronize()
    assert_close(out[..., 4:4 + c], merge(ln.reshape(h.shape)), what="window merge + LayerNorm")
    assert torch.equal(out[..., 4 + 2 * c:4 + 3 * c].cpu(), torch.from_numpy(merge(h)))
    assert bool((out[..., :4] == 7).all()) and bool((out[..., 4 + c:4 + 2 * c] == 7).all())
    assert bool((out[..., 4 + 3 * c:] == 7).all())


@pytest.mark.parametrize("b,grid,win,c", [(2, (40, 40), 20, 384), (3, (8, 12), 4, 64), (1, (6, 6), 3, 1024),
                                          (2, (5, 10), 5, 132)])
def test_window_partition_layernorm(cuda, b, grid, win, c):
    """ko_window_partition_ln: (t + pos) cut into windows led by the class token — bit-exact against the same
    additions in float32 — and its LayerNorm within 1e-5 of float64."""
    gh, gw = grid
    r = np.random.default_rng(c + 3 * win)
    t = (2 * r.standard_normal((b, gh, gw, c)) + 0.3).astype(np.float32)
    pos = (0.5 * r.standard_normal((gh, gw, c))).astype(np.float32)
    cls = r.standard_normal(c).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    bt = (0.1 * r.standard_normal(c)).astype(np.float32)
    v = (t + pos).reshape(b, gh // win, win, gw // win, win, c).transpose(0, 1, 3, 2, 4, 5).reshape(-1, win * win, c)
    ref_h = np.concatenate([np.broadcast_to(cls, (v.shape[0], 1, c)), v], 1)
    _, ref_y = OK.residual_layernorm(ref_h.reshape(-1, c), np.zeros((ref_h.size // c, c), np.float32), None, None,
                                     g, bt, 1e-6)
    tt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    h, y = K.window_partition_layernorm(tt(t), tt(pos), tt(cls), win, tt(g), tt(bt), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(h.cpu(), torch.from_numpy(np.ascontiguousarray(ref_h)))
    assert_close(y, ref_y.reshape(ref_h.shape), what="window partition + LayerNorm")


def test_window_partition_rejects_bad_shapes(cuda):
    t = torch.zeros(1, 8, 8, 64, device=cuda)
    pos, cls, g = torch.zeros(8, 8, 64, device=cuda), torch.zeros(64, device=cuda), torch.ones(64, device=cuda)
    with pytest.raises(ValueError):  # the grid is not a multiple of win
        K.window_partition_layernorm(t, pos, cls, 3, g, g)
    with pytest.raises(ValueError):  # pos of the wrong grid
        K.window_partition_layernorm(t, pos[:4], cls, 4, g, g)
    with pytest.raises(ValueError):  # gamma shorter than C
        K.window_partition_layernorm(t, pos, cls, 4, g[:32].contiguous(), g)
    with pytest.raises(ValueError):  # C not a multiple of 4 (checked by the entry point)
        K.window_partition_layernorm(t[..., :62].contiguous(), pos[..., :62].contiguous(), cls[:62].contiguous(), 4,
                                     g[:62].contiguous(), g[:62].contiguous())


def test_window_merge_rejects_bad_shapes(cuda):
    h = torch.zeros(4, 17, 64, device=cuda)
    out = torch.zeros(1, 8, 8, 64, device=cuda)
    with pytest.raises(ValueError):  # the slice runs past the buffer's channels
        K.window_merge_layernorm(h, (8, 8), 4, out, 4, normalize=False)
    with pytest.raises(ValueError):  # tokens per window do not match win
        K.window_merge_layernorm(h, (8, 8), 3, out, 0, normalize=False)
    with pytest.raises(ValueError):  # normalize without gamma/beta
        K.window_merge_layernorm(h, (8, 8), 4, out, 0)
    g = torch.ones(32, device=cuda)
    with pytest.raises(ValueError):  # gamma / beta shorter than C
        K.window_merge_layernorm(h, (8, 8), 4, out, 0, g, g)


@pytest.mark.parametrize("shape", [(2, 7, 9, 12), (4, 40, 40, 128)])
def test_im2col3x3_matches_padded_shifts(cuda, shape):
    """ko_im2col3x3 is a pure copy: bit-exact against the padded nine-view concatenation."""
    x = torch.randn(*shape, generator=torch.Generator().manual_seed(shape[-1]))
    b, h, w, c = shape
    xp = torch.nn.functional.pad(x, (0, 0, 1, 1, 1, 1))
    ref = torch.cat([xp[:, dy:dy + h, dx:dx + w] for dy in range(3) for dx in range(3)], -1).reshape(b * h * w, 9 * c)
    got = K.im2col3x3(x.to(cuda)).cpu()
    assert torch.equal(got, ref)


# ---------------------------------------------------------------- deformable sampling
def deform_inputs(r, b, row=256, nq=300, nh=16, npts=2):
    value = r.standard_normal((b, 1600, row)).astype(np.float32)
    loc = r.uniform(-0.05, 1.05, (b, nq, nh, 1, npts, 2)).astype(np.float32)
    logits = r.standard_normal((b, nq, nh, npts))
    aw = (np.exp(logits) / np.exp(logits).sum(-1, keepdims=True)).astype(np.float32)
    return value, loc, aw


@pytest.mark.parametrize("b,nq,nh,npts,width", [(2, 300, 16, 2, 96), (3, 37, 4, 4, 50), (1, 1, 1, 1, 3)])
def test_deform_prep(cuda, b, nq, nh, npts, width):
    """ko_deform_prep: loc bit-identical to the reference's float32 arithmetic (model.py:224-225), aw = the point
    softmax within 1e-6."""
    g = torch.Generator().manual_seed(b * 100 + nq)
    oa = (2 * torch.randn(b, nq, width, generator=g)).to(cuda)
    ref = torch.cat([torch.rand(b, nq, 2, generator=g), 0.05 + 0.3 * torch.rand(b, nq, 2, generator=g)], -1).to(cuda)
    loc, aw = K.deform_prep(oa, ref, nh, npts)
    off = oa[..., :nh * npts * 2].reshape(b, nq, nh, npts, 2)
    r = ref[:, :, None, None, :]
    want_loc = r[..., :2] + off / npts * r[..., 2:] * 0.5
    lg = oa[..., nh * npts * 2:nh * npts * 3].reshape(b, nq, nh, npts).double()
    want_aw = torch.softmax(lg, -1)
    torch.cuda.synchronize()
    assert torch.equal(loc, want_loc)
    assert (aw.double() - want_aw).abs().max().item() <= 1e-6


def test_deform_prep_rejects_bad_sizes(cuda):
    oa, ref = torch.zeros(1, 4, 40, device=cuda), torch.zeros(1, 4, 4, device=cuda)
    with pytest.raises(ValueError):  # the row holds fewer than NH * NP * 3 values
        K.deform_prep(oa, ref, 16, 2)
    with pytest.raises(ValueError):  # more than 8 points (checked by the entry point)
        K.deform_prep(torch.zeros(1, 4, 27, device=cuda), ref, 1, 9)


@pytest.mark.parametrize("batch", [1, 3, 64])
def test_deform_attn(cuda, batch):
    r = np.random.default_rng(batch + 11)
    value, loc, aw = deform_inputs(r, batch)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    g = K.deform_attn(t(value), t(loc).reshape(batch, 300, 16, 2, 2), t(aw), (40, 40), 16, 16)
    ref = OK.deform_attn(value, loc.reshape(batch, 300, 16, 2, 2), aw, (40, 40), 16, 16)
    assert_close(g, ref, what="deform")


@pytest.mark.parametrize("offset", [0, 256, 512, 768])
def test_deform_attn_fused_value_layout(cuda, offset):
    r = np.random.default_rng(offset + 5)
    value, loc, aw = deform_inputs(r, 2, row=1024)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    loc = loc.reshape(2, 300, 16, 2, 2)
    g = K.deform_attn(t(value), t(loc), t(aw), (40, 40), 16, 16, offset=offset)
    assert_close(g, OK.deform_attn(value, loc, aw, (40, 40), 16, 16, offset), what=f"offset {offset}")


def test_deform_attn_large_map(cuda):
    """A larger map (80x80 tokens, 4 heads) through the two-point kernel."""
    r = np.random.default_rng(8)
    value = r.standard_normal((2, 80 * 80, 64)).astype(np.float32)
    loc = r.uniform(-0.05, 1.05, (2, 50, 4, 2, 2)).astype(np.float32)
    aw = r.uniform(0, 1, (2, 50, 4, 2)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    g = K.deform_attn(t(value), t(loc), t(aw), (80, 80), 4, 16)
    assert_close(g, OK.deform_attn(value, loc, aw, (80, 80), 4, 16, 0), what="large map")


def test_deform_attn_three_points_odd_shape(cuda):
    """The general 4-channel kernel: 2 chunks per head, 3 points, 37 queries and a non-square map."""
    r = np.random.default_rng(9)
    value = r.standard_normal((3, 13 * 17, 32)).astype(np.float32)
    loc = r.uniform(-0.1, 1.1, (3, 37, 3, 3, 2)).astype(np.float32)
    aw = r.uniform(0, 1, (3, 37, 3, 3)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    g = K.deform_attn(t(value), t(loc), t(aw), (13, 17), 3, 8, offset=4)
    assert_close(g, OK.deform_attn(value, loc, aw, (13, 17), 3, 8, 4), what="three points")


def test_deform_attn_scalar_path(cuda):
    r = np.random.default_rng(3)
    value = r.standard_normal((2, 12 * 7, 45)).astype(np.float32)
    loc = r.uniform(-0.2, 1.2, (2, 9, 5, 3, 2)).astype(np.float32)
    aw = r.uniform(0, 1, (2, 9, 5, 3)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    g = K.deform_attn(t(value), t(loc), t(aw), (12, 7), 5, 7, offset=3)
    assert_close(g, OK.deform_attn(value, loc, aw, (12, 7), 5, 7, 3), what="scalar path")


# ---------------------------------------------------------------- 3xTF32 GEMM
@pytest.mark.parametrize("m,k,n", [(1600, 384, 1536), (4800, 384, 1536), (51200, 384, 1536), (1604, 384, 1152),
                                   (3208, 1536, 384), (6416, 384, 384), (1, 384, 1536), (130, 64, 256),
                                   (1600, 256, 1024), (300, 100, 36), (1000, 768, 384)])
def test_linear_gelu_3xtf32(cuda, m, k, n):
    r = np.random.default_rng(m + k + n)
    x = r.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * r.standard_normal((k, n))).astype(np.float32)
    b = (0.01 * r.standard_normal(n)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    g = K.linear_gelu_f32(t(x), t(w), t(b))
    torch.cuda.synchronize()
    K.check_device_status()
    assert_close(g, OK.linear_gelu_f32(x, w, b), what=f"gemm {m}x{k}x{n}")


def test_linear_gelu_special_values(cuda):
    """The GELU epilogue at the ends of its range, as 0.5 * v * (1 + erf(v / sqrt 2)) gives them: +inf -> +inf,
    -inf -> NaN, large positive v -> v, large negative v -> 0. Powers of two keep the 3xTF32 split exact (lo = 0)."""
    x = torch.zeros(128, 16)
    w = torch.zeros(16, 16)
    x[0, 0], x[1, 0], x[2, 0], x[3, 0], x[4, 0] = 2.0 ** 100, -(2.0 ** 100), 64.0, -64.0, 1.0
    w[0, 0], w[0, 1] = 2.0 ** 100, 1.0  # column 0: x * 2^100 (overflows to +-inf for rows 0, 1); column 1: x
    y = K.linear(x.to(cuda), K.pack_weight(w.to(cuda), torch.zeros(16, device=cuda)), "gelu").cpu()
    assert y[0, 0].item() == float("inf")
    assert math.isnan(y[1, 0].item())
    assert y[0, 1].item() == 2.0 ** 100 and y[2, 1].item() == 64.0
    assert abs(y[1, 1].item()) == 0.0 and abs(y[3, 1].item()) < 1e-30
    assert abs(y[4, 1].item() - 0.8413447460685429) < 1e-6  # GELU(1) = Phi(1)
    assert torch.equal(y[5:], torch.zeros(123, 16))


def test_linear_gelu_split_made_during_capture_is_not_cached(cuda):
    """A weight first seen inside CUDA graph capture: its split exists only once the graph replays, so an eager
    call before the replay must split it again rather than read the graph's unfilled buffer."""
    r = np.random.default_rng(33)
    x = r.standard_normal((512, 384)).astype(np.float32)
    w = (0.02 * r.standard_normal((384, 768))).astype(np.float32)
    b = (0.01 * r.standard_normal(768)).astype(np.float32)
    ref = OK.linear_gelu_f32(x, w, b)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    xd, wd, bd = t(x), t(w), t(b)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            captured = K.linear_gelu_f32(xd, wd, bd)
    eager = K.linear_gelu_f32(xd, wd, bd)            # before any replay
    torch.cuda.synchronize()
    assert_close(eager, ref, what="eager after capture")
    g.replay()
    torch.cuda.synchronize()
    K.check_device_status()
    assert_close(captured, ref, what="replayed graph")
    assert torch.equal(captured, eager)
    del g


@pytest.mark.parametrize("act", [None, "relu"])
def test_linear_packed_acts(cuda, act):
    r = np.random.default_rng(9)
    x = r.standard_normal((777, 256)).astype(np.float32)
    w = r.standard_normal((256, 512)).astype(np.float32)
    b = r.standard_normal(512).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    pw = K.pack_weight(t(w), t(b))
    g = K.linear(t(x), pw, act=act)
    torch.cuda.synchronize()
    K.check_device_status()
    assert_close(g, OK.linear(x, w, b, act), what=str(act))


def test_linear_gelu_workspace_entry_point(cuda):
    """The C-ABI form that packs the weight into a caller-provided workspace on every call."""
    from kernelopt_b200 import _lib
    r = np.random.default_rng(21)
    m, k, n = 3200, 384, 1536
    x = torch.from_numpy(r.standard_normal((m, k)).astype(np.float32)).to(cuda)
    w = torch.from_numpy((0.02 * r.standard_normal((k, n))).astype(np.float32)).to(cuda)
    b = torch.from_numpy((0.01 * r.standard_normal(n)).astype(np.float32)).to(cuda)
    ws = torch.empty(_lib.lib().ko_linear_workspace_bytes(k, n) // 4, dtype=torch.float32, device=cuda)
    out = torch.empty((m, n), dtype=torch.float32, device=cuda)
    _lib.call("ko_linear_gelu_f32", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, k, n, out.data_ptr(),
              ws.data_ptr(), ws.numel() * 4, K.status_word().data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    K.check_device_status()
    assert_close(out, OK.linear_gelu_f32(x.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy()))
    with pytest.raises(ValueError):
        _lib.call("ko_linear_gelu_f32", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, k, n, out.data_ptr(),
                  ws.data_ptr(), 16, None, torch.cuda.current_stream().cuda_stream)


def test_linear_rejects_bad_shapes(cuda):
    x = torch.zeros((10, 6), device=cuda)
    w = torch.zeros((6, 8), device=cuda)
    with pytest.raises(ValueError):
        K.linear_gelu_f32(x, w, torch.zeros(8, device=cuda))
