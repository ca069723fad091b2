"""Query selection on the device (ko_select_queries) against the float64 oracle: the top-NQ proposal indices must
match exactly (descending score, ties by ascending index), the refined reference boxes within 1e-5."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.kernels as OK
from kernelopt_b200 import kernels as K

pytestmark = pytest.mark.gpu


def make(b, n_p, n_c, nq, seed, quantise=None):
    r = np.random.default_rng(seed)
    logits = r.standard_normal((b, n_p, n_c)).astype(np.float32)
    if quantise:
        logits = (np.round(logits / quantise) * quantise).astype(np.float32)  # many exactly tied scores
    delta = (0.2 * r.standard_normal((b, n_p, 4))).astype(np.float32)
    prop = np.concatenate([r.uniform(0, 1, (n_p, 2)), r.uniform(0.01, 0.3, (n_p, 2))], -1).astype(np.float32)
    rp_xy = (0.1 * r.standard_normal((nq, 2))).astype(np.float32)
    rp_ewh = np.exp(0.1 * r.standard_normal((nq, 2))).astype(np.float32)
    return logits, delta, prop, rp_xy, rp_ewh


def run(cuda, logits, delta, prop, rp_xy, rp_ewh, nq):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    ref, idx = K.select_queries(t(logits), t(delta), t(prop), t(rp_xy), t(rp_ewh), nq)
    torch.cuda.synchronize()
    return ref.cpu().double().numpy(), idx.cpu().numpy()


@pytest.mark.parametrize("b,n_p,n_c,nq,quant", [(3, 1600, 11, 300, None), (2, 1600, 11, 300, 0.25),
                                                (1, 37, 5, 37, None), (2, 4096, 3, 1000, None),
                                                (64, 1600, 11, 300, None), (1, 1, 1, 1, None)])
def test_select_matches_oracle(cuda, b, n_p, n_c, nq, quant):
    data = make(b, n_p, n_c, nq, b * 7 + n_p, quant)
    ref_g, idx_g = run(cuda, *data, nq)
    ref_o, idx_o = OK.select_queries(*data, nq)
    assert np.array_equal(idx_g, idx_o), "selected indices or their order differ"
    err = np.abs(ref_g - ref_o).max() / np.abs(ref_o).max()
    assert err <= 1e-5, err


def test_select_ties_order_by_index(cuda):
    """Every score equal: the selection is the first NQ proposals in index order."""
    logits = np.zeros((2, 500, 4), np.float32)
    _, delta, prop, rp_xy, rp_ewh = make(2, 500, 4, 100, 3)
    _, idx = run(cuda, logits, delta, prop, rp_xy, rp_ewh, 100)
    assert np.array_equal(idx, np.tile(np.arange(100), (2, 1)))


def test_select_rejects_bad_sizes(cuda):
    logits, delta, prop, rp_xy, rp_ewh = make(1, 64, 2, 64, 5)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    with pytest.raises(ValueError):  # more queries than proposals
        K.select_queries(t(logits), t(delta), t(prop), t(np.zeros((65, 2), np.float32)),
                         t(np.zeros((65, 2), np.float32)), 65)
    big = make(1, 4097, 1, 10, 6)
    with pytest.raises(ValueError):  # above the 4096 proposals one CTA sorts
        K.select_queries(*(t(a) for a in big), 10)
    with pytest.raises(ValueError):  # delta of the wrong shape
        K.select_queries(t(logits), t(delta[:, :10]), t(prop), t(rp_xy), t(rp_ewh), 64)
