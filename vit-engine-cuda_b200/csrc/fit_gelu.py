"""Derivation of the GELU polynomial in common.cuh (gelu_erf).

GELU(x) = x * Phi(x). With a = |x|, the lower tail is written
    log2 Phi(-a) = g(a) - a^2 / (2 ln 2),   g(a) = log2(Phi(-a) * exp(a^2 / 2)),
and g, smooth and bounded on [0, 5.6], is fitted as g(a) = -1 + a * h(a) with h
of degree 9 (so g(0) = log2(1/2) = -1 exactly), by least squares in the
Chebyshev basis on 200,001 points. Prints the float32 coefficients of h in
Horner order (a^9 first) and the float32 evaluation's error against float64.

    python vit-engine-cuda_b200/csrc/fit_gelu.py
"""
import numpy as np
from scipy.special import log_ndtr, ndtr

A = 5.6
DEG = 9
C2 = 1.0 / (2.0 * np.log(2.0))


def fit():
    a = np.linspace(1e-6, A, 200001)
    g = log_ndtr(-a) / np.log(2.0) + a * a * C2
    t = 2.0 * a / A - 1.0
    V = np.polynomial.chebyshev.chebvander(t, DEG) * a[:, None]
    coef, *_ = np.linalg.lstsq(V, g + 1.0, rcond=None)
    mono = np.polynomial.Polynomial(np.polynomial.chebyshev.cheb2poly(coef))
    return mono(np.polynomial.Polynomial([-1.0, 2.0 / A])).coef.astype(np.float32)


def gelu32(x, co):
    """float32 model of the device code (fma = one rounding; ex2 exact here)."""
    x = x.astype(np.float32)
    a = np.minimum(np.abs(x), np.float32(A))
    h = np.full_like(a, co[-1])
    for c in co[-2::-1]:
        h = (h.astype(np.float64) * a + c).astype(np.float32)
    g = (h.astype(np.float64) * a - 1.0).astype(np.float32)
    s = (x * x).astype(np.float32)
    e = np.exp2((s.astype(np.float64) * np.float64(np.float32(-C2)) + g).astype(np.float32))
    y = (x * e.astype(np.float32)).astype(np.float32)
    return np.where(x > 0, (x - y).astype(np.float32), y)


if __name__ == "__main__":
    co = fit()
    print("h coefficients, a^9 .. a^0:", ", ".join(f"{float(c):.9e}f" for c in co[::-1]))
    x = np.linspace(-8, 8, 1600001).astype(np.float32)
    true = x.astype(np.float64) * ndtr(x.astype(np.float64))
    err = np.abs(gelu32(x, co) - true)
    big = np.abs(true) > 1e-6
    print(f"max relative error (|GELU| > 1e-6): {(err[big] / np.abs(true[big])).max():.2e}")
    print(f"max absolute error: {err.max():.2e}")
