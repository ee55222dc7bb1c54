#!/usr/bin/env python3
"""Generate the polynomial the attention softmax uses for part of its exp2s.

2^x = 2^n * 2^f with n = rint(x) and f = x - n in [-1/2, 1/2]; 2^f is a
polynomial in f fitted for minimum maximum *relative* error on [-1/2, 1/2]
(weighted least squares refined by Lawson's iteratively reweighted least
squares, C. L. Lawson 1961); n is then added to the exponent field.  Printed:
the coefficients c0..cD (lowest degree first) and the maximum relative error
of the polynomial evaluated in float32.

    python exp2_poly.py [--degree 4]
"""
import argparse

import numpy as np


def fit(degree, n=100001, iters=80):
    f = np.linspace(-0.5, 0.5, n)
    y = np.exp2(f)
    v = np.vander(f, degree + 1, increasing=True)
    lw = np.ones_like(f)
    for _ in range(iters):
        sw = np.sqrt(lw) / y
        c, *_ = np.linalg.lstsq(v * sw[:, None], y * sw, rcond=None)
        e = np.abs((v @ c - y) / y)
        lw = lw * e
        lw /= lw.sum()
    return c.astype(np.float32)


def max_rel_error_f32(c):
    f = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    p = np.full_like(f, c[-1])
    for k in range(len(c) - 2, -1, -1):
        p = (p * f + c[k]).astype(np.float32)
    y = np.exp2(f.astype(np.float64))
    return float(np.abs((p - y) / y).max())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--degree", type=int, default=4)
    d = ap.parse_args().degree
    c = fit(d)
    print(f"// degree {d}, max relative error in float32 = {max_rel_error_f32(c):.3g}")
    for k in range(d + 1):
        print(f"{float(c[k]):.9e}f,")


if __name__ == "__main__":
    main()
