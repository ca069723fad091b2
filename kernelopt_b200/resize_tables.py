"""Interpolation tables that make the GPU preprocessing kernel reproduce cv2.resize(INTER_LINEAR) bit for bit.

Same interface as the reference's fast_rfdetr/resize_tables.py:165-184 (`tables`) and :41-43 (`uses_kleidicv`),
plus a `policy` argument: the reference models the macOS arm64 cv2 wheel, which hands the sizes Ballform uses
(1920x1080, 1152x1080, 1280x720 -> 640x640) to KleidiCV; cv2 builds without KleidiCV (the x86-64 wheels) run
OpenCV's own fixed-point path for every size.

    policy="reference"  KleidiCV arithmetic where the reference selects it, OpenCV's elsewhere (the default)
    policy="opencv"     OpenCV's arithmetic for every size (bit-exact with cv2 on x86-64)

The tables are computed by the native library (ko_resize_tables, host code); this module only caches them.
"""
from __future__ import annotations

import ctypes
import functools

import numpy as np

from . import _lib

CH = 3
POLICIES = {"reference": _lib.KO_RESIZE_REFERENCE, "opencv": _lib.KO_RESIZE_OPENCV}


def uses_kleidicv(src_w: int, src_h: int, dst_w: int, dst_h: int) -> bool:
    """True where the modelled cv2 wheel runs KleidiCV (strict downscale, horizontal ratio <= 3)."""
    return (dst_w * 3 >= src_w and dst_w < src_w and dst_h < src_h and dst_w * CH >= 8 and src_w * CH >= 32)


@functools.lru_cache(maxsize=32)
def tables(src_w: int, src_h: int, dst_w: int = 640, dst_h: int = 640, policy: str = "reference"):
    """Returns (mode, xtab int32 [dst_w*3, 4], ytab int32 [dst_h, 4]).

    xtab columns: left element index, right element index, weight a (fx or a0), weight b (0 or a1)
    ytab columns: top row, bottom row, weight (fy or b0), weight (0 or b1)
    The arrays are read-only (they are shared through the cache)."""
    if policy not in POLICIES:
        raise ValueError(f"policy must be one of {sorted(POLICIES)}")
    xt = np.zeros((dst_w * CH, 4), np.int32)
    yt = np.zeros((dst_h, 4), np.int32)
    mode = ctypes.c_int(-1)
    _lib.call("ko_resize_tables", int(src_w), int(src_h), int(dst_w), int(dst_h), POLICIES[policy],
              xt.ctypes.data, yt.ctypes.data, ctypes.byref(mode))
    xt.flags.writeable = False
    yt.flags.writeable = False
    return int(mode.value), xt, yt
