"""CPU oracle (test infrastructure): the reference's cv2.resize table model and preprocessing, in numpy.

Restates fast_rfdetr/resize_tables.py (tables :165-184, KleidiCV x :46-138, KleidiCV y :141-145, OpenCV axis
:148-162, evaluation :187-205), the normalisation LUT of detector.py:70-71 and the kernel's channel handling
(kernels.py:95-102). Written as whole-array numpy where the reference loops, except where the modelled
library itself is sequential (the KleidiCV coordinate stepping).
"""
from __future__ import annotations

import numpy as np

FIXP = 16
HALF = 1 << (FIXP - 1)
CH = 3
MEAN = np.asarray([.485, .456, .406], dtype=np.float32)
STD = np.asarray([.229, .224, .225], dtype=np.float32)


def _rdiv(n, d):
    return (n + d // 2) // d


def _centre(d, src, dst):
    """16.16 source coordinate of destination pixel centre d (resize_tables.py:37-38)."""
    return _rdiv(((np.asarray(d, np.int64) << FIXP) + HALF) * src, dst) - HALF + (1 << (FIXP - 9))


def kleidicv_selected(src_w, src_h, dst_w, dst_h) -> bool:
    """resize_tables.py:41-43."""
    return dst_w * 3 >= src_w and dst_w < src_w and dst_h < src_h and dst_w * CH >= 8 and src_w * CH >= 32


def _kleidi_x(src_w: int, dst_w: int):
    ratio = 2 if src_w / dst_w < 1.8 else 3
    n_el = dst_w * CH
    el = np.zeros(n_el, np.int64)
    fx = np.zeros(n_el, np.int64)
    one = _rdiv(src_w << FIXP, dst_w)
    lanes = np.arange(16)

    def vec(e0, sx, ip):
        k = (ip + lanes) // CH
        ch = (ip + lanes) % CH
        pos = (sx & 0xFFFF) + _rdiv((k * src_w) << FIXP, dst_w)
        lane_px = (pos >> FIXP) & 0xFF
        idx = np.maximum(((lane_px * 3) & 0xFF) - ip, 0) + np.where(k == 0, ch - ip, ch)
        el[e0:e0 + 16] = (sx >> FIXP) * CH + ip + idx
        fx[e0:e0 + 16] = (pos >> 8) & 0xFF

    def scalar(e0, n, ip, sx):
        # element j of the run: pixel p(j) = 0 for the first 3-ip elements, then one pixel per 3 elements
        j = np.arange(n)
        p = np.where(j < CH - ip, 0, (j - (CH - ip)) // CH + 1)
        sxp = sx + p * one
        first = p == 0
        el[e0:e0 + n] = (sxp >> FIXP) * CH + np.where(first, ip + j, (j - (CH - ip)) % CH)
        fx[e0:e0 + n] = (sxp & 0xFFFF) >> 8

    def overrun(e):
        return (int(_centre(e // CH, src_w, dst_w)) >> FIXP) * CH + e % CH + 16 * ratio > src_w * CH

    pairs = n_el // 32 if src_w * CH >= 16 * ratio else 0
    n_vec = 2 * pairs
    n_tail = -(-(n_el - 32 * pairs) // 8)
    e = done = 0
    if n_vec > 3:
        last = n_vec - 1
        while overrun(last * 16):
            last -= 1
            if last <= 0:
                break
        inside = 0 if (last == 0 and overrun(0)) else last + 1
        sx = int(_centre(0, src_w, dst_w))
        five, six = _rdiv((src_w * 5) << FIXP, dst_w), _rdiv((src_w * 6) << FIXP, dst_w)
        for g in range(inside // 3):
            if g % 171 == 170:  # the stepped coordinate is recomputed once every 171 groups
                sx = int(_centre(e // CH, src_w, dst_w))
            vec(e, sx, 0)
            vec(e + 16, sx + five, 1)
            vec(e + 32, sx + 2 * five, 2)
            sx += 2 * five + six
            e += 48
            done += 3
    while done < n_vec:
        scalar(e, 16, e % CH, int(_centre(e // CH, src_w, dst_w)))
        done += 1
        e += 16
    for _ in range(n_tail):
        e = min(e, n_el - 8)
        scalar(e, 8, e % CH, int(_centre(e // CH, src_w, dst_w)))
        e += 8
    return el, fx


def _opencv_axis(src: int, dst: int, clamp: bool):
    f = ((np.arange(dst, dtype=np.float64) + 0.5) * (src / dst) - 0.5).astype(np.float32)
    s = np.floor(f).astype(np.int64)
    frac = (f - s.astype(np.float32)).astype(np.float32)
    if clamp:
        lo, hi = s < 0, s >= src - 1
        frac[lo] = 0
        s[lo] = 0
        frac[hi] = 0
        s[hi] = src - 1
    w1 = np.rint(frac * np.float32(2048)).astype(np.int64)
    w0 = np.rint((np.float32(1) - frac) * np.float32(2048)).astype(np.int64)
    return np.clip(s, 0, src - 1), np.clip(s + 1, 0, src - 1), w0, w1


def tables(src_w: int, src_h: int, dst_w: int = 640, dst_h: int = 640, policy: str = "reference"):
    """(mode, xtab int32 [dst_w*3, 4], ytab int32 [dst_h, 4]) — resize_tables.py:165-184 (+ the opencv policy)."""
    if policy == "reference" and kleidicv_selected(src_w, src_h, dst_w, dst_h):
        el, fx = _kleidi_x(src_w, dst_w)
        sy = _centre(np.arange(dst_h), src_h, dst_h)
        row = sy >> FIXP
        fy = (sy - (row << FIXP)) >> (FIXP - 8)
        xt = np.stack([el, el + CH, fx, np.zeros_like(fx)], 1)
        yt = np.stack([row, np.minimum(row + 1, src_h - 1), fy, np.zeros_like(fy)], 1)
        return 0, xt.astype(np.int32), yt.astype(np.int32)
    x0, x1, a0, a1 = _opencv_axis(src_w, dst_w, True)
    y0, y1, b0, b1 = _opencv_axis(src_h, dst_h, False)
    c = np.tile(np.arange(CH), dst_w)
    xt = np.stack([np.repeat(x0, CH) * CH + c, np.repeat(x1, CH) * CH + c, np.repeat(a0, CH), np.repeat(a1, CH)], 1)
    yt = np.stack([y0, y1, b0, b1], 1)
    return 1, xt.astype(np.int32), yt.astype(np.int32)


def resize(img: np.ndarray, dst_w: int = 640, dst_h: int = 640, policy: str = "reference") -> np.ndarray:
    """uint8 [dst_h, dst_w, 3] BGR: evaluation of the tables (resize_tables.py:187-205)."""
    h, w, _ = img.shape
    mode, xt, yt = tables(w, h, dst_w, dst_h, policy)
    flat = img.reshape(h, w * CH).astype(np.int64)
    top, bot = flat[yt[:, 0]], flat[yt[:, 1]]
    A, B = top[:, xt[:, 0]], top[:, xt[:, 1]]
    C, D = bot[:, xt[:, 0]], bot[:, xt[:, 1]]
    if mode == 0:
        fy, fx = yt[:, 2:3].astype(np.int64), xt[None, :, 2].astype(np.int64)
        left = (A * 256 + (C - A) * fy + 128) >> 8
        right = (B * 256 + (D - B) * fy + 128) >> 8
        v = (left * 256 + (right - left) * fx + 128) >> 8
    else:
        a0, a1 = xt[None, :, 2].astype(np.int64), xt[None, :, 3].astype(np.int64)
        b0, b1 = yt[:, 2:3].astype(np.int64), yt[:, 3:4].astype(np.int64)
        v = ((((A * a0 + B * a1) >> 4) * b0 >> 16) + (((C * a0 + D * a1) >> 4) * b1 >> 16) + 2) >> 2
    return np.clip(v, 0, 255).astype(np.uint8).reshape(dst_h, dst_w, CH)


def lut() -> np.ndarray:
    """float32 [3, 256]: lut[c, v] = (v/255 - mean[c]) / std[c], RGB order, same float32 ops as detector.py:70."""
    t = (np.arange(256, dtype=np.float32)[:, None] / 255. - MEAN) / STD
    return np.ascontiguousarray(t.T)


def normalize(resized_bgr: np.ndarray) -> np.ndarray:
    """float32 HWC RGB from a resized uint8 BGR image (Ballform's preprocessing after the resize)."""
    rgb = resized_bgr[..., ::-1].astype(np.float32) / 255.
    return ((rgb - MEAN) / STD).astype(np.float32)


def preprocess(img: np.ndarray, dst: int = 640, policy: str = "reference", layout: str = "hwc") -> np.ndarray:
    """The preprocessing kernel's output for one frame: 'hwc' [dst,dst,3], 'chw' [3,dst,dst] or 'patch16'."""
    out = normalize(resize(img, dst, dst, policy))
    if layout == "hwc":
        return out
    if layout == "chw":
        return np.ascontiguousarray(out.transpose(2, 0, 1))
    if layout == "patch16":
        g = dst // 16
        return np.ascontiguousarray(out.reshape(g, 16, g, 16, 3).transpose(0, 2, 1, 3, 4).reshape(g * g, 768))
    raise ValueError(layout)
