"""Fit the arcsine polynomial used by devmath.cuh (and restated by the CPU oracle).

With the classic range reduction (Cody & Waite; also Cephes asinf), asin(a) for
a in [0, 1/2] is a + a z P(z), z = a^2, and for a in (1/2, 1] it is
pi/2 - 2 (s + s z P(z)) with z = (1 - a)/2, s = sqrt(z): one polynomial P on
z in [0, 1/4] serves both.  P(z) approximates (asin(sqrt z) - sqrt z) / z^(3/2); its
coefficients come from iteratively reweighted least squares (Lawson's algorithm) towards
the minimax relative error of the final result, then rounded to float32.  Evaluated in
float32 with Horner fused multiply-adds (and sqrt z as z * rsq(z) within 1 ulp) the
result is within 2 ulp of asin (checked below on 2M points of [-1, 1]).

    python zeno_b200/csrc/fit_asin_poly.py
"""
import numpy as np


def fit(deg=4, iters=60, n=4000):
    z = 0.125 * (1 - np.cos(np.linspace(0, np.pi, n)))[1:]  # (0, 1/4]
    a = np.sqrt(z)
    y = (np.arcsin(a) - a) / (a * z)
    V = np.vander(z, deg + 1, increasing=True)
    # weight: the error of the final result a + a z P relative to asin(a)
    scale = (a * z) / np.arcsin(a)
    w = np.ones_like(z)
    for _ in range(iters):
        W = np.sqrt(w)[:, None]
        c, *_ = np.linalg.lstsq(V * scale[:, None] * W, y * scale * np.sqrt(w), rcond=None)
        err = np.abs(V @ c - y) * scale
        w = w * err
        w /= w.sum()
    return c, err.max()


def f32(x):
    return np.asarray(x, dtype=np.float32)


def fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def asin32(x, c32):
    """The kernel's evaluation order in float32 (sqrt correctly rounded here; the kernel's
    z * rsq(z) adds at most one ulp of s)."""
    a = np.abs(x).astype(np.float32)
    small = a <= np.float32(0.5)
    z = np.where(small, (a * a).astype(np.float32), (np.float32(0.5) * (np.float32(1.0) - a)).astype(np.float32))
    s = np.where(small, a, np.sqrt(z.astype(np.float64)).astype(np.float32))
    p = np.full_like(z, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        p = fma32(p, z, np.full_like(z, c32[k]))
    t = fma32((s * z).astype(np.float32), p, s)
    r = np.where(small, t, fma32(np.full_like(t, -2.0), t, np.full_like(t, np.float32(np.pi / 2))))
    return np.where(x < 0, -r, r).astype(np.float32)


def check(c32, npts=2_000_000):
    x = np.random.default_rng(0).uniform(-1, 1, npts).astype(np.float32)
    x = np.concatenate([x, np.array([-1, -0.5, 0, 0.5, 1], np.float32), np.nextafter(f32(0.5), f32(1)).ravel()])
    r = asin32(x, c32)
    ref = np.arcsin(x.astype(np.float64))
    ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    return float(np.max(np.abs(r - ref) / np.maximum(ulp, np.spacing(np.float32(0)))))


if __name__ == "__main__":
    for deg in (3, 4, 5):
        c, e = fit(deg)
        c32 = c.astype(np.float32)
        print(deg, "relative error of the fit:", e, "max ulp (float32):", check(c32))
        print("  coefficients:", [repr(float(v)) for v in c32])
