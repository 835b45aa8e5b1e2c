"""Fit the arctangent polynomial used by devmath.cuh (and restated by the CPU oracle).

atan(a) on [0, 1] is approximated as a * P(a^2), P of degree 8.  The coefficients come
from iteratively reweighted least squares (Lawson's algorithm) towards the minimax
*relative* error on Chebyshev-spaced points, then rounded to float32 with the constant
term pinned to 1.  Evaluated by Horner's rule with fused multiply-adds in float32 the
result is within 1.5 ulp of atan(a) (checked below on 2M random points).

    python zeno_b200/csrc/fit_atan_poly.py
"""
import numpy as np


def fit(deg=8, iters=60, n=4000):
    a = 0.5 * (1 - np.cos(np.linspace(0, np.pi, n)))[1:]
    s = a * a
    y = np.arctan(a) / a
    V = np.vander(s, deg + 1, increasing=True)
    w = np.ones_like(s)
    for _ in range(iters):
        W = np.sqrt(w)[:, None]
        c, *_ = np.linalg.lstsq(V * W / y[:, None], np.sqrt(w), rcond=None)
        err = np.abs(V @ c - y) / y
        w = w * err
        w /= w.sum()
    return c, err.max()


def check(c32, npts=2_000_000):
    def fma32(a, b, c):
        return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)
    a = np.random.default_rng(0).random(npts).astype(np.float32)
    s = (a * a).astype(np.float32)
    p = np.full_like(s, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        p = fma32(p, s, np.full_like(s, c32[k]))
    r = (a * p).astype(np.float32)
    ref = np.arctan(a.astype(np.float64))
    return float(np.max(np.abs(r - ref) / np.spacing(ref.astype(np.float32)).astype(np.float64)))


if __name__ == "__main__":
    c, e = fit()
    c32 = c.astype(np.float32)
    c32[0] = 1.0
    print("relative error of the fit:", e)
    print("coefficients:", [repr(float(x)) for x in c32])
    print("max ulp error (float32 Horner/FMA):", check(c32))
