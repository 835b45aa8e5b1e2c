"""The reproducible arctangent shared (as two separate restatements) by the oracle and the
kernel: within 2 ulp of the correctly rounded value over the whole range, and the
documented special values."""
import ctypes

import numpy as np

from oracle.zeno_oracle import lib


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
