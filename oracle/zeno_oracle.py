"""TEST INFRASTRUCTURE ONLY: ctypes wrapper around the CPU oracle library.

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline / reference leg of
``bench.py`` may import this module.  The product package ``zeno_b200`` never does.

The oracle is a serial C++ restatement of the reference world set-up and step
(see oracle_step.cpp for the per-stage reference citations).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libzeno_oracle.so"


class ZoConfig(ctypes.Structure):
    _fields_ = [
        ("num_envs", ctypes.c_uint32),
        ("timestep", ctypes.c_float),
        ("contact_iterations", ctypes.c_uint32),
        ("max_contacts_per_env", ctypes.c_uint32),
        ("seed", ctypes.c_uint64),
        ("substeps", ctypes.c_uint32),
        ("enable_profiling", ctypes.c_bool),
        ("max_bodies_per_env", ctypes.c_uint32),
        ("max_joints_per_env", ctypes.c_uint32),
        ("max_geoms_per_env", ctypes.c_uint32),
    ]


class ZoTask(ctypes.Structure):
    _fields_ = [
        ("enabled", ctypes.c_uint32),
        ("body", ctypes.c_uint32),
        ("auto_reset", ctypes.c_uint32),
        ("_pad", ctypes.c_uint32),
        ("z_min", ctypes.c_float),
        ("z_max", ctypes.c_float),
        ("noise", ctypes.c_float),
        ("forward_weight", ctypes.c_float),
        ("alive_bonus", ctypes.c_float),
        ("ctrl_cost", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("env_offset", ctypes.c_uint64),
    ]


def build() -> Path:
    """Compile the oracle library with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        vp, f32p, u8p = ctypes.c_void_p, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint8)
        L.zo_create.restype = vp
        L.zo_create.argtypes = [ctypes.c_char_p, ctypes.POINTER(ZoConfig)]
        L.zo_create_ex.restype = vp
        L.zo_create_ex.argtypes = [ctypes.c_char_p, ctypes.POINTER(ZoConfig), ctypes.c_uint32]
        L.zo_destroy.argtypes = [vp]
        L.zo_step.argtypes = [vp, f32p, ctypes.c_uint32]
        L.zo_run.argtypes = [vp, f32p, ctypes.c_uint32, ctypes.c_uint32]
        L.zo_run_threads.argtypes = [vp, f32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        L.zo_step_subset.argtypes = [vp, f32p, u8p, ctypes.c_uint32]
        L.zo_reset.argtypes = [vp, u8p]
        L.zo_reset_to_state.argtypes = [vp, f32p, f32p, f32p, f32p, u8p]
        L.zo_set_gravity.argtypes = [vp, ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.zo_set_timestep.argtypes = [vp, ctypes.c_float]
        L.zo_set_task.argtypes = [vp, ctypes.POINTER(ZoTask)]
        L.zo_dims.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32)]
        L.zo_buffer.restype = vp
        L.zo_buffer.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_size_t)]
        L.zo_set_narrow_mode.argtypes = [vp, ctypes.c_uint32]
        L.zo_set_arithmetic.argtypes = [vp, ctypes.c_uint32]
        L.zo_narrow_cpu.argtypes = [f32p, f32p, f32p, f32p, f32p, ctypes.c_uint32]
        L.zo_gjk_epa.argtypes = [f32p, f32p, f32p, f32p, f32p]
        L.zo_eval_math.argtypes = [ctypes.c_uint32, f32p, f32p, f32p, ctypes.c_uint64]
        _lib = L
    return _lib


CONTACT_DTYPE = np.dtype(
    [("position_pen", "4f4"), ("normal_friction", "4f4"), ("indices", "4u4"), ("impulses", "4f4")]
)


def _fptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _u8ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


class OracleWorld:
    """A world stepped by the CPU oracle; buffers are numpy views into oracle memory."""

    def __init__(self, xml: str, num_envs=1, timestep=0.0, contact_iterations=4,
                 max_contacts_per_env=64, seed=42, substeps=1, semantics="reference",
                 arithmetic="canonical"):
        cfg = ZoConfig(num_envs, timestep, contact_iterations, max_contacts_per_env, seed, substeps,
                       False, 0, 0, 0)
        sem = {"reference": 0, "corrected": 1}[semantics]
        self._h = lib().zo_create_ex(xml.encode(), ctypes.byref(cfg), sem)
        if not self._h:
            raise RuntimeError("oracle world creation failed")
        d = (ctypes.c_uint32 * 10)()
        lib().zo_dims(self._h, d)
        (self.num_envs, self.num_bodies, self.num_joints, self.num_actuators, self.num_geoms,
         self.num_sensors, self.max_contacts, self.num_constraints, self.obs_dim,
         self.num_colors) = list(d)
        if arithmetic != "canonical" and self.set_arithmetic(arithmetic) != 0:
            raise ValueError(f"arithmetic {arithmetic!r} not available for this world")

    def __del__(self):
        if getattr(self, "_h", None):
            lib().zo_destroy(self._h)
            self._h = None

    def raw(self, name: str, dtype=np.float32) -> np.ndarray:
        n = ctypes.c_size_t()
        p = lib().zo_buffer(self._h, name.encode(), ctypes.byref(n))
        if not p or n.value == 0:
            return np.zeros(0, dtype=dtype)
        buf = (ctypes.c_uint8 * n.value).from_address(p)
        return np.frombuffer(buf, dtype=dtype)

    def state(self) -> dict:
        E, B = self.num_envs, self.num_bodies
        J1, O1 = max(self.num_joints, 1), max(self.obs_dim, 1)
        return {
            "positions": self.raw("positions").reshape(E, B, 4).copy(),
            "quaternions": self.raw("quaternions").reshape(E, B, 4).copy(),
            "velocities": self.raw("velocities").reshape(E, B, 4).copy(),
            "angular_velocities": self.raw("angular_velocities").reshape(E, B, 4).copy(),
            "accelerations": self.raw("accelerations").reshape(E, B, 4).copy(),
            "joint_positions": self.raw("joint_positions").reshape(E, J1)[:, : self.num_joints].copy(),
            "joint_velocities": self.raw("joint_velocities").reshape(E, J1)[:, : self.num_joints].copy(),
            "joint_torques": self.raw("joint_torques").reshape(E, J1)[:, : self.num_joints].copy(),
            "observations": self.raw("observations").reshape(E, O1)[:, : self.obs_dim].copy(),
            "rewards": self.raw("rewards").copy(),
            "dones": self.raw("dones", np.uint8).copy(),
            "contacts": self.raw("contacts", CONTACT_DTYPE).reshape(E, self.max_contacts).copy(),
            "contact_counts": self.raw("contact_counts", np.uint32).copy(),
        }

    def step(self, actions: np.ndarray, substeps: int = 0) -> None:
        a = np.ascontiguousarray(actions, dtype=np.float32).ravel()
        lib().zo_step(self._h, _fptr(a), substeps)

    def run(self, actions: np.ndarray, substeps: int = 0, threads: int = 1) -> None:
        """actions: (nsteps, E, A); environments split across `threads` host threads."""
        a = np.ascontiguousarray(actions, dtype=np.float32)
        lib().zo_run_threads(self._h, _fptr(a), a.shape[0], substeps, threads)

    def step_subset(self, actions, mask, substeps=0):
        a = np.ascontiguousarray(actions, dtype=np.float32).ravel()
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        lib().zo_step_subset(self._h, _fptr(a), _u8ptr(m), substeps)

    def reset(self, mask=None):
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        lib().zo_reset(self._h, _u8ptr(m))

    def reset_to_state(self, pos, quat, vel=None, angvel=None, mask=None):
        cv = lambda x: None if x is None else np.ascontiguousarray(x, dtype=np.float32)
        pos, quat, vel, angvel = cv(pos), cv(quat), cv(vel), cv(angvel)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        lib().zo_reset_to_state(self._h, _fptr(pos), _fptr(quat), _fptr(vel), _fptr(angvel), _u8ptr(m))

    def set_gravity(self, g):
        lib().zo_set_gravity(self._h, *map(float, g))

    def set_timestep(self, ts):
        return lib().zo_set_timestep(self._h, float(ts))

    def set_task(self, enabled=True, body=1, z_min=-np.inf, z_max=np.inf, auto_reset=False, noise=0.0,
                 forward_weight=1.0, alive_bonus=1.0, ctrl_cost=0.01, seed=0, env_offset=0):
        t = ZoTask(int(enabled), body, int(auto_reset), 0, z_min, z_max, noise, forward_weight,
                   alive_bonus, ctrl_cost, seed, env_offset)
        return lib().zo_set_task(self._h, ctypes.byref(t))

    def set_narrow_phase(self, mode: int) -> int:
        """0: the reference's GPU narrow phase (default); 1: its CPU detectCollision; 2: as 1,
        plus GJK + EPA for box-capsule pairs."""
        return lib().zo_set_narrow_mode(self._h, int(mode))

    def set_arithmetic(self, mode: str) -> int:
        """'canonical': the arithmetic the product kernel evaluates bit for bit (default);
        'literal': the reference Metal kernels' own expressions in plain IEEE single precision
        (oracle_literal.cpp), for tolerance checks of the canonical arithmetic;
        'contracted': the literal source compiled with FMA contraction (the spread of the
        reference's own source under two legitimate compilations)."""
        return lib().zo_set_arithmetic(self._h, {"canonical": 0, "literal": 1, "contracted": 2}[mode])

    def model_table(self, name: str) -> bytes:
        return self.raw(name, np.uint8).tobytes()


def narrow_cpu(geom_a, body_a, geom_b, body_b, mode=1):
    """detectCollision of the restated CPU collision code for two geoms (mode 2: with GJK +
    EPA for box-capsule pairs).  geom_*: (type, lx, ly, lz, size0, size1, size2); body_*:
    (px, py, pz, qx, qy, qz, qw).  Returns None or (point[3], normal[3], penetration)."""
    ga, gb = (np.asarray(g, np.float32) for g in (geom_a, geom_b))
    ba, bb = (np.asarray(b, np.float32) for b in (body_a, body_b))
    out = np.zeros(7, np.float32)
    if not lib().zo_narrow_cpu(_fptr(ga), _fptr(ba), _fptr(gb), _fptr(bb), _fptr(out), int(mode)):
        return None
    return out[:3].copy(), out[3:6].copy(), float(out[6])


def gjk_epa(geom_a, body_a, geom_b, body_b):
    """The reference's GJK then EPA (src/collision/gjk.zig) on two shapes (types 0 sphere,
    1 capsule, 2 box; arguments as narrow_cpu).  Returns (intersect, epa) with epa None or
    (normal[3], depth, point_a[3], point_b[3])."""
    ga, gb = (np.asarray(g, np.float32) for g in (geom_a, geom_b))
    ba, bb = (np.asarray(b, np.float32) for b in (body_a, body_b))
    out = np.zeros(10, np.float32)
    r = lib().zo_gjk_epa(_fptr(ga), _fptr(ba), _fptr(gb), _fptr(bb), _fptr(out))
    if r < 2:
        return bool(r), None
    return True, (out[:3].copy(), float(out[3]), out[4:7].copy(), out[7:10].copy())


def eval_math(fn, x, y=None):
    """The oracle's canonical scalar function `fn` (0 rsq, 1 rcp, 2 atan2(x, y), 3 asin,
    4 len((x, y, x/2))) over an array."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    yy = None if y is None else np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty_like(x)
    if lib().zo_eval_math(fn, _fptr(x), _fptr(yy), _fptr(out), x.size) != 0:
        raise ValueError("bad arguments")
    return out
