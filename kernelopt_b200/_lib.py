"""ctypes binding of libkernelopt.so, the C ABI declared in include/kernelopt.h.

The library is built in-tree (kernelopt_b200/build.py) and loaded from this package directory only. There is no
fallback: if the library is missing or the device is not an sm_100 GPU, the calls raise.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libkernelopt.so")

KO_OK = 0
KO_ERR_INVALID_ARGUMENT = 1001
KO_ERR_UNSUPPORTED = 1002
KO_ERR_DEVICE_TIMEOUT = 1003

KO_LAYOUT_HWC, KO_LAYOUT_CHW, KO_LAYOUT_PATCH16 = 0, 1, 2
KO_RESIZE_REFERENCE, KO_RESIZE_OPENCV = 0, 1
KO_ACT_NONE, KO_ACT_GELU, KO_ACT_RELU, KO_ACT_SILU = 0, 1, 2, 3

_i64, _i32, _f32, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p


class ImageDesc(ctypes.Structure):
    """Mirror of ko_image_desc."""
    _fields_ = [("src", _vp), ("xtab", _vp), ("ytab", _vp), ("src_h", _i64), ("src_w", _i64),
                ("src_stride", _i64), ("mode", ctypes.c_int32), ("_pad", ctypes.c_int32)]


# name -> (restype, argtypes); every symbol include/kernelopt.h declares
SIGNATURES = {
    "ko_last_error_string": (ctypes.c_char_p, []),
    "ko_abi_version": (_i32, []),
    "ko_check_device": (_i32, []),
    "ko_resize_tables": (_i32, [_i64, _i64, _i64, _i64, _i32, _vp, _vp, ctypes.POINTER(_i32)]),
    "ko_preprocess": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _i64, _i32, _vp, _vp]),
    "ko_preprocess_batch": (_i32, [ctypes.POINTER(ImageDesc), _i32, _vp, _i64, _i32, _vp, _vp]),
    "ko_residual_layernorm": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _vp, _vp, _vp]),
    "ko_deform_attn": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "ko_linear_workspace_bytes": (_i64, [_i64, _i64]),
    "ko_pack_weight_tf32x3": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "ko_linear_f32_packed": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp]),
    "ko_linear_gelu_f32": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "ko_linear_gelu_f32_noalloc": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "ko_attention_f32": (_i32, [_vp, _vp, _vp, _vp] + [_i64] * 12 + [_f32, _vp, _vp]),
    "ko_layernorm": (_i32, [_vp, _vp, _vp, _f32, _i64, _i64, _i32, _vp, _vp]),
    "ko_linear_residual_ln_f32_packed": (_i32, [_vp] * 7 + [_f32, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _vp, _vp]),
    "ko_conv3x3_ln_f32_packed": (_i32, [_vp, _i64] + [_vp] * 4 + [_f32] + [_i64] * 5 + [_i32, _vp, _i64, _vp, _vp]),
    "ko_wait_probe": (_i32, [_i64, _vp, _vp]),
    "ko_window_merge_ln": (_i32, [_vp, _vp, _vp, _f32] + [_i64] * 5 + [_i32, _vp, _i64, _i64, _vp]),
    "ko_window_partition_ln": (_i32, [_vp] * 5 + [_f32] + [_i64] * 5 + [_vp, _vp, _vp]),
    "ko_deform_prep": (_i32, [_vp, _vp] + [_i64] * 5 + [_vp, _vp, _vp]),
    "ko_select_queries": (_i32, [_vp] * 5 + [_i64] * 4 + [_vp, _vp, _vp]),
    "ko_im2col3x3": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "ko_linear_add_f32_packed": (_i32, [_vp] * 4 + [_i64] * 5 + [_i32, _vp, _vp, _vp]),
    "ko_sine_embed": (_i32, [_vp, _vp, _i64, _vp, _vp]),
    "ko_linear_small_f32": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp]),
    "ko_box_head_f32": (_i32, [_vp] * 4 + [_i64, _i64, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class KernelError(RuntimeError):
    """A libkernelopt entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Loads libkernelopt.so once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m kernelopt_b200.build`")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = res, args
                _lib = handle
    return _lib


# Kernel-launching entry points, counted per call (bench.py reports launches per step from these counts).
LAUNCHING = {"ko_preprocess": 1, "ko_preprocess_batch": 1, "ko_residual_layernorm": 1, "ko_deform_attn": 1,
             "ko_pack_weight_tf32x3": 1, "ko_linear_f32_packed": 1, "ko_linear_gelu_f32": 2,
             "ko_linear_gelu_f32_noalloc": 2, "ko_attention_f32": 1, "ko_layernorm": 1, "ko_im2col3x3": 1,
             "ko_linear_residual_ln_f32_packed": 1, "ko_select_queries": 1,
             "ko_conv3x3_ln_f32_packed": 1,
             "ko_wait_probe": 1, "ko_window_merge_ln": 1, "ko_window_partition_ln": 1, "ko_deform_prep": 1,
             "ko_linear_add_f32_packed": 1, "ko_sine_embed": 1, "ko_linear_small_f32": 1, "ko_box_head_f32": 1}
launch_count: dict[str, int] = {}


def call(name: str, *args) -> int:
    """Calls entry point `name`; raises KernelError on a non-zero status."""
    if name in LAUNCHING:
        launch_count[name] = launch_count.get(name, 0) + LAUNCHING[name]
    st = getattr(lib(), name)(*args)
    if st != KO_OK:
        msg = lib().ko_last_error_string().decode(errors="replace")
        if st == KO_ERR_INVALID_ARGUMENT:
            raise ValueError(f"{name}: {msg}")
        raise KernelError(name, st, msg)
    return st
