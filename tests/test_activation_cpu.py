"""The erf approximation of the tensor-core builds' GEMM and DConv epilogues
(erf_as in demucs-wgpu_b200/csrc/common.cuh: Abramowitz & Stegun, Handbook of
Mathematical Functions, eq. 7.1.26) restated here with the same constants:
it stays within the published bound of 1.5e-7 of erf in exact arithmetic, and
within 1e-6 when evaluated in f32 (the device's exponential and reciprocal
are approximate too; the epilogues' inputs carry tf32 rounding, 2^-11
relative, far above either); GELU built on it stays
within 2e-7 |x| of the exact GELU. The device results are checked end to end
by the tensor-core builds' parity tests."""

import math

import numpy as np

P, A = 0.3275911, (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def erf_as(z, dtype):
    z = np.asarray(z, dtype)
    a = np.abs(z)
    t = dtype(1) / (dtype(1) + dtype(P) * a)
    q = dtype(A[4])
    for c in A[3::-1]:
        q = q * t + dtype(c)
    r = dtype(1) - q * t * np.exp(-a * a).astype(dtype)
    return np.copysign(r, z)


def test_erf_as_meets_the_published_bound():
    z = np.linspace(-6.0, 6.0, 240001)
    exact = np.array([math.erf(v) for v in z])
    assert np.max(np.abs(erf_as(z, np.float64) - exact)) <= 1.5e-7
    z32 = z.astype(np.float32)
    exact32 = np.array([math.erf(float(v)) for v in z32])
    assert np.max(np.abs(erf_as(z32, np.float32) - exact32)) <= 1e-6
    assert np.array_equal(erf_as(-z, np.float64), -erf_as(z, np.float64))
    assert erf_as(np.array([40.0, -40.0]), np.float32).tolist() == [1.0, -1.0]


def test_gelu_on_erf_as_tracks_the_exact_gelu():
    x = np.linspace(-12.0, 12.0, 48001)
    exact = 0.5 * x * (1.0 + np.array([math.erf(v / math.sqrt(2.0)) for v in x]))
    approx = 0.5 * x * (1.0 + erf_as(x / math.sqrt(2.0), np.float64))
    assert np.all(np.abs(approx - exact) <= 2e-7 * np.maximum(np.abs(x), 1e-3) + 1e-12)
