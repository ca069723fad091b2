"""CPU oracle (test infrastructure): float64 numpy restatements of the three fp32 hot-path kernels.

Each follows the reference's unfused semantics (the path model.py takes with fused=False) and the reference
kernel's argument conventions (fast_rfdetr/kernels.py). Inputs may be float32; all arithmetic is float64.
Parity unpinned at the MLX boundary: the reference's own MLX path cannot run here and ships no golden vectors
for these kernels.
"""
from __future__ import annotations

import math

import numpy as np
from scipy.special import erf


def residual_layernorm(h, o, bias, scale, gamma, beta, eps):
    """(h + (o + bias) * scale, LayerNorm of that) — kernels.py:53-67, model.py:140-141 with the bias of
    model.py:139 and mx.fast.layer_norm (biased variance, eps inside the square root)."""
    h, o = np.asarray(h, np.float64), np.asarray(o, np.float64)
    b = 0.0 if bias is None else np.asarray(bias, np.float64)
    s = 1.0 if scale is None else np.asarray(scale, np.float64)
    h_out = h + (o + b) * s
    mean = h_out.mean(-1, keepdims=True)
    var = ((h_out - mean) ** 2).mean(-1, keepdims=True)
    y = (h_out - mean) / np.sqrt(var + eps) * np.asarray(gamma, np.float64) + np.asarray(beta, np.float64)
    return h_out, y


def gelu_erf(v):
    """0.5 v (1 + erf(v / sqrt 2)) — model.py:143."""
    return 0.5 * v * (1.0 + erf(v / math.sqrt(2.0)))


def linear(x, w, bias=None, act=None):
    """x @ w + bias, then the activation ('gelu', 'relu' or None) — model.py:75-78 and :142-143."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    if act == "gelu":
        y = gelu_erf(y)
    elif act == "relu":
        y = np.maximum(y, 0.0)
    return y


def linear_gelu_f32(x, w, bias):
    """GELU_erf(x @ w + bias) — kernels.py:271-285."""
    return linear(x, w, bias, "gelu")


def linear_residual_layernorm(x, w, bias, scale, resid, gamma, beta, eps, act=None):
    """The GEMM followed by residual_layernorm, as the reference runs them one after the other: the attention
    out-projection / fc2 GEMM, then h + (o + bias) * scale and its LayerNorm (model.py:121-123, 129-132,
    kernels.py:53-67); without a residual and with act='silu', the projector's conv GEMM -> channel LayerNorm ->
    SiLU (model.py:148-158). Returns (h_out, y)."""
    o = linear(x, w)
    h = np.zeros_like(o) if resid is None else np.asarray(resid, np.float64)
    h_out, y = residual_layernorm(h, o, bias, scale, gamma, beta, eps)
    if act == "silu":
        y = y / (1.0 + np.exp(-y))
    return h_out, y


def deform_attn(value, loc, aw, grid_hw, nh, hd, offset=0):
    """out[b,q,h*hd+d] = sum_p aw * bilinear(value[b, :, offset + h*hd + d] as GH x GW, loc) — kernels.py:165-181
    and model.py:196-216 + 228-229 (GridSample, zero padding, align_corners=False).

    value [B, GH*GW, ROW]; loc [B, NQ, NH, NP, 2]; aw [B, NQ, NH, NP] -> [B, NQ, NH*hd]."""
    value = np.asarray(value, np.float64)
    loc = np.asarray(loc, np.float64)
    aw = np.asarray(aw, np.float64)
    b, n_tok, _ = value.shape
    gh, gw = grid_hw
    nq, npts = loc.shape[1], loc.shape[3]
    v = value[:, :, offset:offset + nh * hd].reshape(b, n_tok, nh, hd)          # [B, T, NH, HD]
    x = loc[..., 0] * gw - 0.5
    y = loc[..., 1] * gh - 0.5
    x0, y0 = np.floor(x), np.floor(y)
    fx, fy = x - x0, y - y0
    bi = np.arange(b)[:, None, None, None]
    hi = np.arange(nh)[None, None, :, None]
    out = np.zeros((b, nq, nh, npts, hd))
    for dy, wy in ((0, 1 - fy), (1, fy)):
        for dx, wx in ((0, 1 - fx), (1, fx)):
            xi, yi = (x0 + dx).astype(np.int64), (y0 + dy).astype(np.int64)
            ok = (xi >= 0) & (xi < gw) & (yi >= 0) & (yi < gh)
            tok = np.clip(yi, 0, gh - 1) * gw + np.clip(xi, 0, gw - 1)             # [B, NQ, NH, NP]
            g = v[bi, tok, hi]                                                      # [B, NQ, NH, NP, HD]
            out += g * np.where(ok, wx * wy, 0.0)[..., None]
    return (out * aw[..., None]).sum(axis=3).reshape(b, nq, nh * hd)


def select_queries(logits, delta, proposals, rp_xy, rp_ewh, nq):
    """model.py:175-185 after the two heads: score = max over classes, coord = refined proposal, the nq best
    proposals by a stable descending sort (ties by ascending index), ref = the selected coords refined by the
    query reference points. Returns (ref [B, nq, 4] float64, idx [B, nq])."""
    logits = np.asarray(logits, np.float64)
    delta = np.asarray(delta, np.float64)
    prop = np.asarray(proposals, np.float64)
    scores = logits.max(-1)
    coord = np.concatenate([delta[..., :2] * prop[:, 2:] + prop[:, :2], np.exp(delta[..., 2:]) * prop[:, 2:]], -1)
    idx = np.argsort(-np.asarray(logits, np.float32).max(-1), axis=-1, kind="stable")[:, :nq]
    ts = np.take_along_axis(coord, idx[..., None], axis=1)
    rxy, rwh = np.asarray(rp_xy, np.float64), np.asarray(rp_ewh, np.float64)
    return np.concatenate([rxy * ts[..., 2:] + ts[..., :2], rwh * ts[..., 2:]], -1), idx
