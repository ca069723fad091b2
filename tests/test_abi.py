"""The C ABI library loads, exports every symbol include/kernelopt.h declares, and rejects bad arguments on the
host before touching the GPU (no compute calls here: these run without a GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from kernelopt_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kernelopt.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(ko_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert len(names) >= 12
    assert set(names) == set(_lib.SIGNATURES), "ctypes bindings and header disagree"


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared():
        assert hasattr(lib, name), name


def test_abi_version_and_error_string():
    assert _lib.lib().ko_abi_version() == 2
    assert isinstance(_lib.lib().ko_last_error_string(), bytes)


@pytest.mark.parametrize("call", [
    ("ko_residual_layernorm", (1, 1, None, None, 1, 1, 1e-6, 10, 3, 1, 1, None)),          # C % 4 != 0
    ("ko_deform_attn", (1, 1, 1, 1, 300, 16, 16, 2, 40, 40, 200, 0, 1, None)),              # NH*HD > ROW
    ("ko_linear_f32_packed", (16, 16, None, 8, 6, 8, 0, 16, None, None)),                   # K % 4 != 0
    ("ko_linear_f32_packed", (16, 16, None, 8, 8, 8, 7, 16, None, None)),                   # unknown act
    ("ko_linear_gelu_f32", (16, 16, 16, 8, 8, 8, 16, 16, 4, None, None)),                   # workspace small
    ("ko_pack_weight_tf32x3", (16, 0, 8, 16, None)),                                        # K = 0
    ("ko_linear_gelu_f32_noalloc", (16, 16, None, 8, 1 << 20, 1 << 20, 16, None, None)),    # K*N over the scratch
    ("ko_linear_residual_ln_f32_packed",
     (16, 16, None, None, None, 16, 16, 1e-6, 128, 256, 256, 99, None, 16, 0, None, None)),  # unknown act
    ("ko_linear_residual_ln_f32_packed",
     (16, 16, None, None, None, None, None, 1e-6, 128, 256, 256, 0, None, 16, 0, None, None)),  # no gamma/beta
    ("ko_linear_residual_ln_f32_packed",
     (16, 16, None, None, None, 16, 16, 1e-6, 128, 256, 256, 0, None, 32, 250, None, None)),  # ldy < N
    ("ko_conv3x3_ln_f32_packed", (16, 0, 16, 16, 16, 16, 1e-6, 1, 8, 8, 8, 256, 0, 32, 0, None, None)),  # C % 16
    ("ko_conv3x3_ln_f32_packed", (16, 0, 16, 16, 16, 16, 1e-6, 1, 8, 8, 16, 256, 0, 16, 0, None, None)),  # y is x
    ("ko_conv3x3_ln_f32_packed", (16, 18, 16, 16, 16, 16, 1e-6, 1, 8, 8, 16, 256, 0, 32, 0, None, None)),  # ldx
    ("ko_linear_add_f32_packed", (16, 16, None, 16, 512, 6, 8, 8, 8, 0, 32, None, None)),    # add_cols % 4
    ("ko_linear_add_f32_packed", (16, 16, None, 20, 512, 8, 8, 8, 8, 0, 32, None, None)),    # addend unaligned
    ("ko_linear_add_f32_packed", (16, 16, None, 16, 8, 12, 8, 8, 8, 0, 32, None, None)),     # add_cols > N
    ("ko_linear_small_f32", (16, 16, None, 8, 256, 40, 0, 16, None)),                         # N > 32
    ("ko_linear_small_f32", (16, 16, None, 8, 256, 11, 1, 16, None)),                         # GELU not offered
    ("ko_box_head_f32", (16, 16, None, 20, 8, 256, 16, None)),                                # ref unaligned
    ("ko_sine_embed", (16, 16, 10, 20, None)),                                                # out unaligned
    ("ko_attention_f32", (16, 16, 16, 16, 1, 128, 1, 48, 0, 48, 0, 48, 0, 48, 0, 48, 0.125, None, None)),  # HD 48
    ("ko_attention_f32", (16, 16, 16, 16, 1, 128, 1, 32, 0, 30, 0, 32, 0, 32, 0, 32, 0.125, None, None)),  # stride
    ("ko_layernorm", (16, 16, 16, 1e-6, 10, 6, 0, 16, None)),                                # C % 4 != 0
    ("ko_layernorm", (16, 16, 16, 1e-6, 10, 8, 1, 16, None)),                                # GELU not offered
    ("ko_window_merge_ln", (16, 16, 16, 1e-6, 1, 8, 8, 4, 64, 1, 16, 64, 4, None)),          # col_off + C > ldo
    ("ko_window_merge_ln", (16, None, None, 1e-6, 1, 8, 8, 4, 64, 1, 16, 64, 0, None)),      # normalize, no gamma
    ("ko_window_partition_ln", (16, 16, 16, 16, 16, 1e-6, 1, 8, 8, 3, 64, 16, 16, None)),    # H % win != 0
    ("ko_window_partition_ln", (20, 16, 16, 16, 16, 1e-6, 1, 8, 8, 4, 64, 16, 16, None)),    # t unaligned
    ("ko_deform_prep", (16, 16, 1, 300, 16, 9, 432, 16, 16, None)),                          # NP > 8
    ("ko_deform_prep", (16, 16, 1, 300, 16, 4, 100, 16, 16, None)),                          # row < NH*NP*3
    ("ko_deform_prep", (16, 20, 1, 300, 16, 4, 192, 16, 16, None)),                          # ref unaligned
    ("ko_deform_prep", (16, 16, 1, 300, 1 << 20, 1, 3 << 20, 16, 16, None)),                 # NH > 4096
    ("ko_select_queries", (16, 16, 16, 16, 16, 1, 100, 2, 300, 16, 16, None)),               # NQ > NP
    ("ko_select_queries", (16, 16, 16, 16, 16, 1, 5000, 2, 300, 16, 16, None)),              # NP > 4096
    ("ko_im2col3x3", (16, 1, 8, 8, 6, 16, None)),                                            # C % 4 != 0
    ("ko_im2col3x3", (20, 1, 8, 8, 8, 16, None)),                                            # x unaligned
    ("ko_preprocess", (16, 720, 1280, 3840, 16, 16, 16, 2, 640, 0, 16, None)),               # mode 2
    ("ko_preprocess", (16, 720, 1280, 100, 16, 16, 16, 0, 640, 0, 16, None)),                # stride < 3 W
    ("ko_preprocess", (16, 720, 1280, 3840, 16, 16, 16, 0, 648, 2, 16, None)),               # PATCH16, dst % 16
    ("ko_preprocess", (16, 720, 1280, 3840, 16, 16, 16, 0, 640, 5, 16, None)),               # unknown layout
])
def test_invalid_arguments_are_rejected_on_the_host(call):
    name, args = call
    with pytest.raises(ValueError):
        _lib.call(name, *args)
    assert _lib.lib().ko_last_error_string()


def test_preprocess_batch_rejects_empty_and_oversized():
    with pytest.raises(ValueError):
        _lib.call("ko_preprocess_batch", None, 0, 16, 640, 0, 16, None)
    descs = (_lib.ImageDesc * 65)()
    with pytest.raises(ValueError):
        _lib.call("ko_preprocess_batch", descs, 65, 16, 640, 0, 16, None)


def test_linear_workspace_size():
    assert _lib.lib().ko_linear_workspace_bytes(384, 1536) == 2 * 384 * 1536 * 4


@pytest.mark.parametrize("call", [
    ("ko_linear_f32_packed", (16, 16, None, 256, 384, 1536, 0, 16, None, None)),
    ("ko_linear_gelu_f32", (16, 16, 16, 256, 384, 1536, 16, 16, 2 * 384 * 1536 * 4, None, None)),
    ("ko_linear_residual_ln_f32_packed",
     (16, 16, None, None, None, 16, 16, 1e-6, 512, 384, 256, 0, None, 32, 0, None, None)),
    ("ko_conv3x3_ln_f32_packed", (16, 0, 16, 16, 16, 16, 1e-6, 1, 8, 8, 16, 256, 0, 32, 0, None, None)),
    ("ko_linear_add_f32_packed", (16, 16, None, 32, 512, 256, 256, 384, 768, 0, 48, None, None)),
    ("ko_linear_small_f32", (16, 16, None, 300, 256, 11, 0, 32, None)),
    ("ko_box_head_f32", (16, 16, None, 32, 300, 256, 48, None)),
    ("ko_attention_f32", (16, 16, 16, 32, 1, 128, 1, 64, 0, 64, 0, 64, 0, 64, 0, 64, 0.125, None, None)),
    ("ko_im2col3x3", (16, 1, 8, 8, 8, 32, None)),
])
def test_valid_calls_without_a_device_fail_cleanly(call):
    """With no usable CUDA device the SM count is unknown: a well-formed call must return KO_ERR_UNSUPPORTED with
    a message before it sizes a grid (no division by a zero SM count, no zero-block launch)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    name, args = call
    with pytest.raises(_lib.KernelError) as e:
        _lib.call(name, *args)
    assert e.value.status == _lib.KO_ERR_UNSUPPORTED
    assert _lib.lib().ko_last_error_string()


def test_check_device_reports_a_missing_gpu():
    """Without a CUDA device the device check fails cleanly (KO_ERR_UNSUPPORTED and a message) on every call."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    for _ in range(2):
        assert _lib.lib().ko_check_device() == _lib.KO_ERR_UNSUPPORTED
        assert b"sm_100a" in _lib.lib().ko_last_error_string()
