"""Failure detection of the kernels with on-chip waits, exercised without a GPU fault: ko_wait_probe runs the
same bounded mbarrier wait on a barrier that nothing completes. The wait must give up after its limit, a second
warp must leave on the CTA's abort flag, the status word must carry KO_ERR_DEVICE_TIMEOUT (raised on the host by
check_device_status), and the context must stay usable."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle.kernels as OK
from kernelopt_b200 import _lib
from kernelopt_b200 import kernels as K

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    word = K.status_word(cuda)
    word.zero_()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.call("ko_wait_probe", 20_000_000, word.data_ptr(), torch.cuda.current_stream().cuda_stream)  # 20 ms
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(word.item()) == _lib.KO_ERR_DEVICE_TIMEOUT
    with pytest.raises(_lib.KernelError):
        K.check_device_status(cuda)
    assert int(word.item()) == 0  # cleared by the check
    # the second warp left on the abort flag, not on its own 2 s limit
    assert elapsed < 1.0, elapsed
    # the context still runs kernels correctly
    r = np.random.default_rng(0)
    x = r.standard_normal((300, 64)).astype(np.float32)
    w = (0.1 * r.standard_normal((64, 128))).astype(np.float32)
    b = (0.1 * r.standard_normal(128)).astype(np.float32)
    g = K.linear(torch.from_numpy(x).to(cuda), K.pack_weight(torch.from_numpy(w).to(cuda), torch.from_numpy(b).to(cuda)))
    torch.cuda.synchronize()
    K.check_device_status(cuda)
    ref = OK.linear(x, w, b)
    assert np.abs(g.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


def test_wait_probe_rejects_bad_limits(cuda):
    word = K.status_word(cuda)
    with pytest.raises(ValueError):
        _lib.call("ko_wait_probe", -1, word.data_ptr(), None)
    with pytest.raises(ValueError):
        _lib.call("ko_wait_probe", 1000, None, None)
