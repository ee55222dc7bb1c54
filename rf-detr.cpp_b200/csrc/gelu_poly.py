#!/usr/bin/env python3
"""Generate the polynomial used by the GEMM epilogue's erf-GELU.

GELU(x) = 0.5 x (1 + erf(x / sqrt 2)) is rewritten as

    GELU(x) = max(x, 0) - h(|x|),   h(a) = 0.5 a erfc(a / sqrt 2)
            = max(x, 0) - a * exp(-a^2 / 2) * R(a),
    R(a)    = 0.5 * erfcx(a / sqrt 2)

(erfcx(z) = exp(z^2) erfc(z), the scaled complementary error function).
R is smooth and slowly varying on [0, 6], so a low-degree polynomial fits
it; the error that matters is the absolute error of h, i.e. the fit is
weighted by a * exp(-a^2 / 2).  Arguments are clamped to a <= 6, where
h(6) < 7e-9, so the clamp itself is below the fit error.

Method: weighted least squares on a dense grid, refined into a near-minimax
fit by Lawson's iteratively reweighted least squares (C. L. Lawson,
"Contributions to the theory of linear least maximum approximation", 1961).
The reference values come from scipy.special.erfcx.  The printed table holds
-R's coefficients (the epilogue folds the subtraction into its last FMA),
highest degree first, plus the measured maximum |error| of h evaluated in
float32 with exp2.

    python gelu_poly.py [--degree 10]
"""
import argparse

import numpy as np
from scipy.special import erfc, erfcx

A_MAX = 6.0


def fit(degree, n=200001, iters=60):
    a = np.linspace(0.0, A_MAX, n)
    r = 0.5 * erfcx(a / np.sqrt(2.0))
    w = np.maximum(a * np.exp(-0.5 * a * a), 1e-12)
    v = np.vander(a / A_MAX, degree + 1, increasing=True)
    lw = np.ones_like(a)
    for _ in range(iters):
        sw = np.sqrt(lw) * w
        c, *_ = np.linalg.lstsq(v * sw[:, None], r * sw, rcond=None)
        e = np.abs(w * (v @ c - r))
        lw = lw * e
        lw /= lw.sum()
    return (c / A_MAX ** np.arange(degree + 1)).astype(np.float32)


def max_error_f32(coef):
    a = np.linspace(0.0, A_MAX, 200001).astype(np.float32)
    p = np.full_like(a, coef[-1])
    for k in range(len(coef) - 2, -1, -1):
        p = (p * a + coef[k]).astype(np.float32)
    e = np.exp2((a * np.float32(-0.5 / np.log(2.0))) * a).astype(np.float32)
    h = (a * e * p).astype(np.float32)
    ref = 0.5 * a.astype(np.float64) * erfc(a.astype(np.float64) / np.sqrt(2.0))
    return float(np.abs(h - ref).max())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--degree", type=int, default=10)
    d = ap.parse_args().degree
    c = fit(d)
    print(f"// degree {d}, max |h error| in float32 = {max_error_f32(c):.3g}")
    for k in range(d, -1, -1):
        print(f"{-float(c[k]):.9e}f,")


if __name__ == "__main__":
    main()
