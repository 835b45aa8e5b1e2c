"""The canonical scalar functions shared (as two separate restatements) by the oracle and
the kernels: the reproducible arctangent (within 3 ulp of the correctly rounded value over
the whole range, documented special values) and the Newton-Raphson reciprocal and
reciprocal square root (within 1 ulp over every binade of their domain), plus a GPU test
that the kernels' versions equal the oracle's bit for bit, inside and outside that
domain."""
import ctypes

import numpy as np
import pytest

from oracle.zeno_oracle import eval_math, lib


def _fn(name):
    f = getattr(lib(), name)
    f.restype = ctypes.c_float
    return f


def ulp_err(got, ref):
    ref32 = ref.astype(np.float32)
    return np.abs(got.astype(np.float64) - ref) / np.spacing(np.abs(ref32)).astype(np.float64)


def test_atan2_accuracy():
    f = _fn("zo_atan2")
    rng = np.random.default_rng(0)
    y = (rng.standard_normal(20000) * 10 ** rng.uniform(-3, 3, 20000)).astype(np.float32)
    x = (rng.standard_normal(20000) * 10 ** rng.uniform(-3, 3, 20000)).astype(np.float32)
    got = np.array([f(ctypes.c_float(a), ctypes.c_float(b)) for a, b in zip(y, x)], dtype=np.float32)
    ref = np.arctan2(y.astype(np.float64), x.astype(np.float64))
    assert ulp_err(got, ref).max() <= 3.0


def test_asin_accuracy():
    f = _fn("zo_asin")
    xs = np.linspace(-1, 1, 20001).astype(np.float32)
    got = np.array([f(ctypes.c_float(v)) for v in xs], dtype=np.float32)
    ref = np.arcsin(xs.astype(np.float64))
    err = np.abs(got - ref)
    assert err.max() < 1e-6 + 4 * np.spacing(np.float32(1.57))


def test_special_values():
    f = _fn("zo_atan2")
    assert f(ctypes.c_float(0.0), ctypes.c_float(0.0)) == 0.0
    assert abs(f(ctypes.c_float(0.0), ctypes.c_float(-1.0)) - np.pi) < 1e-6
    assert abs(f(ctypes.c_float(1.0), ctypes.c_float(0.0)) - np.pi / 2) < 1e-6
    assert abs(f(ctypes.c_float(-1.0), ctypes.c_float(0.0)) + np.pi / 2) < 1e-6
    assert np.isnan(f(ctypes.c_float(np.nan), ctypes.c_float(1.0)))
    assert np.isnan(f(ctypes.c_float(1.0), ctypes.c_float(np.nan)))


def binade_sweep(n_per=2048, lo=-126, hi=127, seed=0):
    """n_per random mantissas in every binade 2^lo .. 2^hi, plus the powers of two."""
    rng = np.random.default_rng(seed)
    m = rng.uniform(1.0, 2.0, size=(hi - lo + 1, n_per))
    e = np.arange(lo, hi + 1, dtype=np.float64)[:, None]
    x = (m * np.exp2(e)).astype(np.float32).ravel()
    return np.concatenate([x, np.exp2(np.arange(lo, hi + 1)).astype(np.float32)])


def test_rsq_accuracy():
    x = binade_sweep()
    got = eval_math(0, x)
    ref = 1.0 / np.sqrt(x.astype(np.float64))
    assert ulp_err(got, ref).max() <= 1.0


def test_rcp_accuracy():
    x = binade_sweep(lo=-126, hi=124)  # domain: |x| < 2^125
    x = np.concatenate([x, -x])
    got = eval_math(1, x)
    ref = 1.0 / x.astype(np.float64)
    assert ulp_err(got, ref).max() <= 1.0


def test_length_accuracy():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(50000) * 10 ** rng.uniform(-6, 6, 50000)).astype(np.float32)
    y = (rng.standard_normal(50000) * 10 ** rng.uniform(-6, 6, 50000)).astype(np.float32)
    got = eval_math(4, x, y)
    x64, y64 = x.astype(np.float64), y.astype(np.float64)
    ref = np.sqrt(x64 * x64 + y64 * y64 + 0.25 * x64 * x64)
    assert ulp_err(got, ref).max() <= 4.0


def test_newton_special_values():
    z = np.array([0.0], np.float32)
    assert np.isfinite(eval_math(0, z)[0]) and eval_math(0, z)[0] > 1e19  # rsq(0): large, finite
    assert eval_math(4, z, z)[0] == 0.0                       # |0| = 0
    nan = np.array([np.nan], np.float32)
    assert np.isnan(eval_math(0, nan)[0]) and np.isnan(eval_math(1, nan)[0])


def math_inputs():
    rng = np.random.default_rng(7)
    x = binade_sweep(n_per=8192)
    xs = np.concatenate([x, -x, np.array([0.0, -0.0, np.inf, -np.inf, np.nan], np.float32)])
    ys = rng.permutation(xs)
    u = rng.uniform(-1.0, 1.0, 200000).astype(np.float32)
    return xs, ys, np.concatenate([u, np.array([-1.0, 1.0, 0.0, -0.0], np.float32)])


@pytest.mark.gpu
@pytest.mark.parametrize("fn", [0, 1, 2, 3, 4])
def test_gpu_math_equals_oracle(fn):
    """rsq, rcp, atan2, asin and len on the GPU (zeno_eval_math) equal the oracle's bit for
    bit over every binade, both signs and the special values (a NaN result is a NaN on
    both sides; its payload is the hardware's: 0x7fffffff on the GPU, the input's on x86)."""
    from zeno_b200 import _ffi
    xs, ys, u = math_inputs()
    if fn == 3:
        x, y = u, None
    elif fn in (2, 4):
        x, y = xs, ys
    else:
        x, y = xs, None
    a = _ffi.eval_math(fn, x, y)
    b = eval_math(fn, x, y)
    same = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
    assert same.all(), f"{int((~same).sum())} results differ, first input {x[np.argmin(same)]}"

