"""zeno_world_reset_to_state_noalloc, called through the C ABI.

Callers that cannot allocate device memory (their HBM is already reserved by another
allocator, or an allocation must not block or fail mid-episode) use this entry point:
it stages host arrays through a fixed static device array instead of cudaMallocAsync.
Its results must equal zeno_world_reset_to_state's bit for bit, on two calls in a row
(the static array keeps the previous call's contents), and it must refuse worlds larger
than its capacity with a clear error.  This file is collected last on purpose; it passes
both alone in a fresh process and after the other tests."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "zeno_b200" / "lib" / "libzeno.so"
CAPACITY = 1 << 20  # float4 bodies in the static staging array


@pytest.fixture(scope="module")
def capi():
    L = ctypes.CDLL(str(LIB))
    f32p, u8p = ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint8)
    for name in ("zeno_world_reset_to_state", "zeno_world_reset_to_state_noalloc"):
        fn = getattr(L, name)
        fn.argtypes = [ctypes.c_void_p, f32p, f32p, f32p, f32p, u8p]
        fn.restype = ctypes.c_int
    L.zeno_last_error.restype = ctypes.c_char_p
    return L


def handle(world):
    from zeno_b200._ffi import ffi
    return int(ffi.cast("uintptr_t", world.handle))


def fptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def u8ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def state(w):
    return [w.get_body_positions(zero_copy=False), w.get_body_quaternions(zero_copy=False),
            w.get_body_velocities(zero_copy=False), w.get_body_angular_velocities(zero_copy=False),
            w.get_contact_counts()]


def test_noalloc_matches_reset_to_state_twice(capi):
    from zeno_b200 import ZenoWorld, scenes
    E = 64
    a = ZenoWorld(mjcf_string=scenes.ant(), num_envs=E, substeps=4)
    b = ZenoWorld(mjcf_string=scenes.ant(), num_envs=E, substeps=4)
    rng = np.random.default_rng(17)
    acts = rng.uniform(-1, 1, size=(3, E, 8)).astype(np.float32)
    for s in range(3):
        a.step(acts[s])
        b.step(acts[s])
    B = a.num_bodies
    calls = [
        (None, True, True),                                             # every env, all four arrays
        ((np.arange(E) % 3 == 0).astype(np.uint8), False, True),        # masked, no velocities
    ]
    for k, (mask, with_vel, with_ang) in enumerate(calls):
        pos = rng.uniform(-1, 1, (E, B, 4)).astype(np.float32)
        quat = rng.standard_normal((E, B, 4)).astype(np.float32)
        vel = rng.uniform(-1, 1, (E, B, 4)).astype(np.float32) if with_vel else None
        ang = rng.uniform(-1, 1, (E, B, 4)).astype(np.float32) if with_ang else None
        assert capi.zeno_world_reset_to_state(handle(a), fptr(pos), fptr(quat), fptr(vel), fptr(ang), u8ptr(mask)) == 0
        assert capi.zeno_world_reset_to_state_noalloc(handle(b), fptr(pos), fptr(quat), fptr(vel), fptr(ang),
                                                      u8ptr(mask)) == 0
        for x, y in zip(state(a), state(b)):
            assert np.array_equal(np.ascontiguousarray(x).view(np.uint8), np.ascontiguousarray(y).view(np.uint8)), k
        a.step(acts[0])  # and the worlds keep stepping identically
        b.step(acts[0])
        for x, y in zip(state(a), state(b)):
            assert np.array_equal(np.ascontiguousarray(x).view(np.uint8), np.ascontiguousarray(y).view(np.uint8)), k


def test_noalloc_rejects_worlds_beyond_capacity(capi):
    from zeno_b200 import ZenoWorld, scenes
    xml = scenes.pendulum()  # 3 bodies
    E = CAPACITY // 3 + 1
    w = ZenoWorld(mjcf_string=xml, num_envs=E, max_contacts_per_env=1)
    pos = np.zeros((E, 3, 4), np.float32)
    rc = capi.zeno_world_reset_to_state_noalloc(handle(w), fptr(pos), fptr(pos), None, None, None)
    assert rc == -6
    assert b"exceeds the static staging capacity" in capi.zeno_last_error()
