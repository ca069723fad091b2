"""ko_linear_gelu_f32_noalloc: the GEMM+GELU entry point for callers that cannot allocate device memory at run
time (an application allocator that owns all GPU memory, a per-frame real-time path where cudaMalloc/cudaFree
may synchronise the device, a plugin host that passes only inputs and outputs). Its weight-split scratch lives
in the library's static device memory, so the caller provides no workspace.

Checked through the C ABI against the workspace entry point ko_linear_gelu_f32, within the kernel tolerance of
the other tests (max-norm relative error <= 1e-5), on two calls in a row — the second with a different shape,
so it runs on what the first call left in the shared static array. This file is collected last on purpose.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from kernelopt_b200 import _lib

pytestmark = pytest.mark.gpu

REL = 1e-5


def _with_workspace(x, w, b, out, m, k, n, stream):
    ws = torch.empty(_lib.lib().ko_linear_workspace_bytes(k, n) // 4, dtype=torch.float32, device=x.device)
    _lib.call("ko_linear_gelu_f32", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, k, n, out.data_ptr(),
              ws.data_ptr(), ws.numel() * 4, None, stream)
    return ws


def test_noalloc_matches_workspace_entry_point_two_calls(cuda):
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for m, k, n, seed in [(3200, 384, 1536, 1), (777, 256, 512, 2)]:
        r = np.random.default_rng(seed)
        x = torch.from_numpy(r.standard_normal((m, k)).astype(np.float32)).to(cuda)
        w = torch.from_numpy((0.02 * r.standard_normal((k, n))).astype(np.float32)).to(cuda)
        b = torch.from_numpy((0.01 * r.standard_normal(n)).astype(np.float32)).to(cuda)
        ref = torch.empty((m, n), dtype=torch.float32, device=cuda)
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
        ws = _with_workspace(x, w, b, ref, m, k, n, stream)
        _lib.call("ko_linear_gelu_f32_noalloc", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, k, n, got.data_ptr(),
                  status.data_ptr(), stream)
        torch.cuda.synchronize()
        del ws
        assert int(status.item()) == 0
        assert bool(torch.isfinite(got).all())
        err = float((got.double() - ref.double()).abs().max() / ref.double().abs().max())
        assert err <= REL, f"{m}x{k}x{n}: {err:.2e}"


def test_noalloc_rejects_weights_beyond_the_static_scratch(cuda):
    k, n = 1024, 1028                       # K*N = 1,052,672 > KO_NOALLOC_MAX_WEIGHT_ELEMS (1,048,576)
    x = torch.zeros((8, k), device=cuda)
    w = torch.zeros((k, n), device=cuda)
    b = torch.zeros(n, device=cuda)
    out = torch.zeros((8, n), device=cuda)
    with pytest.raises(ValueError, match="KO_NOALLOC_MAX_WEIGHT_ELEMS"):
        _lib.call("ko_linear_gelu_f32_noalloc", x.data_ptr(), w.data_ptr(), b.data_ptr(), 8, k, n, out.data_ptr(),
                  None, torch.cuda.current_stream().cuda_stream)
