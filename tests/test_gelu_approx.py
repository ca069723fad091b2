"""The GELU formulation the GEMM epilogue uses, restated in numpy and checked against math.erf on the CPU.

The epilogue computes GELU(v) = v * Phi(v) with Phi from Abramowitz & Stegun 7.1.26: for x = |v| / sqrt 2,
erfc(x) ~ t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-x^2), t = 1 / (1 + p x), absolute error below 1.5e-7;
q = erfc(x) / 2, Phi(v) = 1 - q for v >= 0 and q for v < 0. This checks the folded constants and the sign
handling of that formulation (in float64, and in float32 as the kernel evaluates it); the CUDA code itself is
checked against float64 GEMM + erf references on the GPU (tests/test_kernels_gpu.py).
"""
from __future__ import annotations

import math

import numpy as np

P, A = 0.3275911, (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def gelu_as(v: np.ndarray, dtype) -> np.ndarray:
    v = v.astype(dtype)
    c = lambda x: dtype(x)  # noqa: E731
    ax = np.abs(v)
    t = c(1.0) / (c(P * 0.7071067811865476) * ax + c(1.0))
    poly = c(0.5 * A[4])
    for a in (A[3], A[2], A[1], A[0]):
        poly = poly * t + c(0.5 * a)
    poly = poly * t
    with np.errstate(over="ignore", under="ignore"):
        e = np.exp2(v * v * c(-0.7213475204444817))
    q = poly * e
    with np.errstate(invalid="ignore"):  # -inf * 0 -> NaN, as 0.5 * v * (1 + erf(v / sqrt 2)) gives
        vq = v * q
        return np.where(v >= 0, np.where(q > 0, v - vq, v), vq)


def gelu_exact(v: np.ndarray) -> np.ndarray:
    return np.array([0.5 * x * (1.0 + math.erf(x / math.sqrt(2.0))) for x in v.astype(np.float64)])


def test_phi_error_bound_float64():
    v = np.linspace(-12.0, 12.0, 200001)
    ref = gelu_exact(v)
    got = gelu_as(v, np.float64)
    # |GELU error| = |v| * |Phi error| <= |v| * 0.75e-7 (half the erfc bound)
    assert np.all(np.abs(got - ref) <= np.abs(v) * 0.75e-7 + 1e-300)


def test_float32_evaluation_within_gemm_tolerance():
    v = np.linspace(-12.0, 12.0, 200001).astype(np.float32)
    ref = gelu_exact(v)
    got = gelu_as(v, np.float32).astype(np.float64)
    err = np.abs(got - ref)
    assert err.max() <= 1e-6 * np.abs(ref).max()  # far inside the 1e-5 normwise bar of the GEMM tests
    assert np.all(err <= np.abs(v) * 4e-7 + 1e-30)


def test_ends_of_the_range():
    v = np.array([np.inf, -np.inf, 1e30, -1e30, 64.0, -64.0, 0.0], dtype=np.float32)
    got = gelu_as(v, np.float32)
    assert got[0] == np.inf and np.isnan(got[1])
    assert got[2] == np.float32(1e30) and got[3] == 0.0
    assert got[4] == 64.0 and abs(got[5]) < 1e-30 and got[6] == 0.0
