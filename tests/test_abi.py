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
    assert _lib.lib().ko_abi_version() == 1
    assert isinstance(_lib.lib().ko_last_error_string(), bytes)


@pytest.mark.parametrize("call", [
    ("ko_residual_layernorm", (1, 1, None, None, 1, 1, 1e-6, 10, 3, 1, 1, None)),          # C % 4 != 0
    ("ko_deform_attn", (1, 1, 1, 1, 300, 16, 16, 2, 40, 40, 200, 0, 1, None)),              # NH*HD > ROW
    ("ko_linear_f32_packed", (16, 16, None, 8, 6, 8, 0, 16, None, None)),                   # K % 4 != 0
    ("ko_linear_f32_packed", (16, 16, None, 8, 8, 8, 7, 16, None, None)),                   # unknown act
    ("ko_linear_gelu_f32", (16, 16, 16, 8, 8, 8, 16, 16, 4, None, None)),                   # workspace small
    ("ko_pack_weight_tf32x3", (16, 0, 8, 16, None)),                                        # K = 0
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
