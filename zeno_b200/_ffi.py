"""cffi binding of libzeno.so and the ``ZenoWorld`` class.

``ZenoWorld`` keeps the reference's Python interface (python/zeno/_ffi.py:439-1162 in
Lulzx/zeno): same constructor arguments, same method names, shapes, dtypes, zero-copy
semantics and error behaviour (RuntimeError on a non-zero return code).  The library
underneath is the sm_100a implementation; its state lives in CUDA managed memory, so
the numpy views returned here alias the buffers the GPU steps.

The native library is required: there is no CPU fallback, and importing this module
raises if libzeno.so cannot be loaded (build it with ``python -m zeno_b200.build``).
"""
from __future__ import annotations

import os
import weakref
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import cffi
import numpy as np

ffi = cffi.FFI()
ffi.cdef("""
    typedef void* ZenoWorldHandle;
    typedef struct {
        uint32_t num_envs; float timestep; uint32_t contact_iterations; uint32_t max_contacts_per_env;
        uint64_t seed; uint32_t substeps; bool enable_profiling;
        uint32_t max_bodies_per_env; uint32_t max_joints_per_env; uint32_t max_geoms_per_env;
    } ZenoConfig;
    typedef struct {
        uint32_t num_envs; uint32_t num_bodies; uint32_t num_joints; uint32_t num_actuators;
        uint32_t num_sensors; uint32_t num_geoms; uint32_t obs_dim; uint32_t action_dim;
        float timestep; uint64_t memory_usage; uint64_t gpu_memory_usage; bool metal_available;
    } ZenoInfo;
    typedef struct {
        float integrate_ns; float collision_broad_ns; float collision_narrow_ns;
        float constraint_solve_ns; float total_step_ns; uint32_t num_contacts; uint32_t num_active_constraints;
    } ZenoProfilingData;
    typedef struct {
        uint32_t enabled; uint32_t body; uint32_t auto_reset; uint32_t _pad;
        float z_min; float z_max; float noise; float forward_weight; float alive_bonus; float ctrl_cost;
        uint64_t seed; uint64_t env_offset;
    } ZenoTaskConfig;

    ZenoWorldHandle zeno_world_create(const char* mjcf_path, const ZenoConfig* config);
    ZenoWorldHandle zeno_world_create_from_string(const char* mjcf_string, const ZenoConfig* config);
    ZenoWorldHandle zeno_world_create_ex(const char* mjcf_path, const ZenoConfig* config, uint32_t semantics);
    ZenoWorldHandle zeno_world_create_from_string_ex(const char* mjcf_string, const ZenoConfig* config,
                                                     uint32_t semantics);
    void zeno_world_destroy(ZenoWorldHandle world);
    int zeno_world_step(ZenoWorldHandle world, const float* actions, uint32_t substeps);
    int zeno_world_step_subset(ZenoWorldHandle world, const float* actions, const uint8_t* env_mask, uint32_t substeps);
    int zeno_world_reset(ZenoWorldHandle world, const uint8_t* env_mask);
    int zeno_world_reset_to_state(ZenoWorldHandle world, const float* positions, const float* quaternions,
                                  const float* velocities, const float* angular_velocities, const uint8_t* env_mask);
    float* zeno_world_get_observations(ZenoWorldHandle world);
    float* zeno_world_get_rewards(ZenoWorldHandle world);
    uint8_t* zeno_world_get_dones(ZenoWorldHandle world);
    float* zeno_world_get_body_positions(ZenoWorldHandle world);
    float* zeno_world_get_body_quaternions(ZenoWorldHandle world);
    float* zeno_world_get_body_velocities(ZenoWorldHandle world);
    float* zeno_world_get_body_angular_velocities(ZenoWorldHandle world);
    float* zeno_world_get_body_accelerations(ZenoWorldHandle world);
    float* zeno_world_get_joint_positions(ZenoWorldHandle world);
    float* zeno_world_get_joint_velocities(ZenoWorldHandle world);
    float* zeno_world_get_joint_forces(ZenoWorldHandle world);
    void* zeno_world_get_contacts(ZenoWorldHandle world);
    uint32_t* zeno_world_get_contact_counts(ZenoWorldHandle world);
    float* zeno_world_get_sensor_data(ZenoWorldHandle world);
    int zeno_world_set_body_positions(ZenoWorldHandle world, const float* positions, const uint8_t* env_mask);
    int zeno_world_set_body_velocities(ZenoWorldHandle world, const float* velocities, const uint8_t* env_mask);
    int zeno_world_set_gravity(ZenoWorldHandle world, float gx, float gy, float gz);
    int zeno_world_set_timestep(ZenoWorldHandle world, float timestep);
    uint32_t zeno_world_num_envs(ZenoWorldHandle world);
    uint32_t zeno_world_num_bodies(ZenoWorldHandle world);
    uint32_t zeno_world_num_joints(ZenoWorldHandle world);
    uint32_t zeno_world_num_sensors(ZenoWorldHandle world);
    uint32_t zeno_world_obs_dim(ZenoWorldHandle world);
    uint32_t zeno_world_action_dim(ZenoWorldHandle world);
    int zeno_world_get_info(ZenoWorldHandle world, ZenoInfo* info);
    int zeno_world_get_profiling(ZenoWorldHandle world, ZenoProfilingData* data);
    void zeno_world_reset_profiling(ZenoWorldHandle world);
    const char* zeno_version();
    bool zeno_metal_available();
    const char* zeno_error_string(int error_code);
    uint64_t zeno_world_memory_usage(ZenoWorldHandle world);
    void zeno_world_compact_memory(ZenoWorldHandle world);
    uint32_t zeno_world_max_contacts_per_env(ZenoWorldHandle world);

    int zeno_world_step_async(ZenoWorldHandle world, const float* actions, uint32_t substeps);
    int zeno_world_synchronize(ZenoWorldHandle world);
    void* zeno_world_get_stream(ZenoWorldHandle world);
    int zeno_world_set_stream(ZenoWorldHandle world, void* cuda_stream);
    int zeno_world_device(ZenoWorldHandle world);
    float* zeno_world_get_observations_device(ZenoWorldHandle world);
    float* zeno_world_get_rewards_device(ZenoWorldHandle world);
    uint8_t* zeno_world_get_dones_device(ZenoWorldHandle world);
    int zeno_world_set_task(ZenoWorldHandle world, const ZenoTaskConfig* task);
    int zeno_world_set_narrow_phase(ZenoWorldHandle world, uint32_t mode);
    uint32_t zeno_world_get_narrow_phase(ZenoWorldHandle world);
    int zeno_world_set_broad_phase(ZenoWorldHandle world, uint32_t mode);
    uint32_t zeno_world_get_broad_phase(ZenoWorldHandle world);
    int zeno_world_set_launch(ZenoWorldHandle world, int lanes, int envs_per_block);
    int zeno_world_get_launch(ZenoWorldHandle world, int* lanes, int* envs_per_block);
    const void* zeno_world_model_table(ZenoWorldHandle world, const char* name, uint64_t* nbytes);
    const char* zeno_last_error(void);
    int zeno_world_get_stage_cycles(ZenoWorldHandle world, double* out, uint32_t n);
    void* zeno_model_create_from_string(const char* mjcf_string);
    int zeno_eval_math(uint32_t fn, const float* x, const float* y, float* out, uint64_t n);
    void* zeno_model_create_from_string_ex(const char* mjcf_string, uint32_t semantics);
    void zeno_model_destroy(void* model);
    const void* zeno_model_table(void* model, const char* name, uint64_t* nbytes);
""")

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libzeno.so"
CONTACT_DTYPE = np.dtype([("position_pen", "4f4"), ("normal_friction", "4f4"), ("indices", "4u4"),
                          ("impulses", "4f4")])


def _load():
    path = Path(os.environ.get("ZENO_B200_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(f"libzeno.so not found at {path}; build it with `python -m zeno_b200.build`")
    return ffi.dlopen(str(path))


_lib = _load()


def version() -> str:
    return ffi.string(_lib.zeno_version()).decode()


def is_metal_available() -> bool:
    """Reference name kept: True when a CUDA device is usable."""
    return bool(_lib.zeno_metal_available())


is_cuda_available = is_metal_available


class ZeroCopyArray:
    """A numpy view of world memory that remembers its world (reference _ffi.py:370-437)."""

    __slots__ = ("_array", "_world_ref", "_ptr")

    def __init__(self, array: np.ndarray, world: "ZenoWorld", ptr):
        self._array, self._world_ref, self._ptr = array, weakref.ref(world), ptr

    @property
    def array(self) -> np.ndarray:
        if self._world_ref() is None:
            raise RuntimeError("World has been destroyed")
        return self._array

    def __array__(self, dtype=None, copy=None):
        return self.array if dtype is None else self.array.astype(dtype)

    def __getattr__(self, name):
        return getattr(self._array, name)

    def __getitem__(self, key):
        return self._array[key]

    def __setitem__(self, key, value):
        self._array[key] = value

    def __len__(self):
        return len(self._array)

    def __repr__(self):
        return f"ZeroCopyArray({self._array.shape}, dtype={self._array.dtype})"

    def copy(self) -> np.ndarray:
        return self._array.copy()

    def is_valid(self) -> bool:
        return self._world_ref() is not None


class CudaArray:
    """Device view of world memory exposing ``__cuda_array_interface__`` (for
    ``torch.as_tensor(x, device="cuda")`` / CuPy without copies)."""

    def __init__(self, ptr: int, shape, typestr: str, owner: "ZenoWorld"):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


SEMANTICS = {"reference": 0, "corrected": 1}


def eval_math(fn: int, x: np.ndarray, y: Optional[np.ndarray] = None) -> np.ndarray:
    """The step kernels' canonical scalar function `fn` (0 rsq, 1 rcp, 2 atan2(x, y),
    3 asin, 4 len((x, y, x/2))) evaluated on the GPU."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    yy = None if y is None else np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty_like(x)
    yp = ffi.NULL if yy is None else ffi.cast("float*", yy.ctypes.data)
    _check(_lib.zeno_eval_math(fn, ffi.cast("float*", x.ctypes.data), yp, ffi.cast("float*", out.ctypes.data),
                               x.size), "Evaluate math")
    return out


def model_tables(mjcf_string: str, semantics: str = "reference") -> Dict[str, bytes]:
    """Build the model on the host only (no GPU) and return its reference-layout tables."""
    h = _lib.zeno_model_create_from_string_ex(mjcf_string.encode(), SEMANTICS[semantics])
    if h == ffi.NULL:
        raise RuntimeError("model build failed: " + ffi.string(_lib.zeno_last_error()).decode())
    try:
        out = {}
        n = ffi.new("uint64_t*")
        for name in ("bodies", "joints", "geoms", "actuators", "sensors", "constraints", "color_ranges", "pairs"):
            p = _lib.zeno_model_table(h, name.encode(), n)
            out[name] = bytes(ffi.buffer(p, n[0])) if p != ffi.NULL and n[0] else b""
        return out
    finally:
        _lib.zeno_model_destroy(h)


def _check(code: int, what: str):
    if code != 0:
        raise RuntimeError(f"{what} failed with error code {code}")


def _f32ptr(a: np.ndarray):
    return ffi.cast("float*", a.ctypes.data)


def _u8ptr(a: Optional[np.ndarray]):
    return ffi.NULL if a is None else ffi.cast("uint8_t*", a.ctypes.data)


class ZenoWorld:
    """A batch of environments stepped on one GPU.

    Parameters follow the reference ``ZenoWorld`` (mjcf_path or mjcf_string, num_envs,
    timestep (0: MJCF value), contact_iterations, max_contacts_per_env, seed, substeps,
    enable_profiling, max_*_per_env).  The world binds to the current CUDA device.
    ``semantics="corrected"`` (no counterpart in the reference) loads and steps the model
    with the MJCF compiler rules and contact conventions the reference skips; the default
    "reference" reproduces the reference, quirks included.
    """

    def __init__(self, mjcf_path: Optional[str] = None, mjcf_string: Optional[str] = None, num_envs: int = 1,
                 timestep: float = 0, contact_iterations: int = 4, max_contacts_per_env: int = 64,
                 seed: int = 42, substeps: int = 1, enable_profiling: bool = False,
                 max_bodies_per_env: int = 64, max_joints_per_env: int = 64, max_geoms_per_env: int = 128,
                 semantics: str = "reference"):
        if mjcf_path is None and mjcf_string is None:
            raise ValueError("Either mjcf_path or mjcf_string must be provided")
        cfg = ffi.new("ZenoConfig*")
        cfg.num_envs, cfg.timestep, cfg.contact_iterations = num_envs, timestep, contact_iterations
        cfg.max_contacts_per_env, cfg.seed, cfg.substeps = max_contacts_per_env, seed, substeps
        cfg.enable_profiling = enable_profiling
        cfg.max_bodies_per_env, cfg.max_joints_per_env, cfg.max_geoms_per_env = (
            max_bodies_per_env, max_joints_per_env, max_geoms_per_env)
        if semantics not in SEMANTICS:
            raise ValueError(f"semantics must be one of {sorted(SEMANTICS)}")
        if mjcf_path is not None:
            self._handle = _lib.zeno_world_create_ex(str(mjcf_path).encode(), cfg, SEMANTICS[semantics])
        else:
            self._handle = _lib.zeno_world_create_from_string_ex(mjcf_string.encode(), cfg, SEMANTICS[semantics])
        if self._handle == ffi.NULL:
            msg = ffi.string(_lib.zeno_last_error()).decode()
            raise RuntimeError("Failed to create Zeno world" + (f": {msg}" if msg else ""))
        info = ffi.new("ZenoInfo*")
        _lib.zeno_world_get_info(self._handle, info)
        self._num_envs, self._obs_dim, self._action_dim = info.num_envs, info.obs_dim, info.action_dim
        self._num_bodies, self._num_joints = info.num_bodies, info.num_joints
        self._num_sensors, self._num_geoms = info.num_sensors, info.num_geoms
        self._timestep, self._memory_usage, self._gpu_memory_usage = (
            info.timestep, info.memory_usage, info.gpu_memory_usage)
        self._max_contacts_per_env = _lib.zeno_world_max_contacts_per_env(self._handle)
        self._cached_arrays: Dict[str, ZeroCopyArray] = {}

    def __del__(self):
        h = getattr(self, "_handle", None)
        try:
            if h is not None and h != ffi.NULL:
                _lib.zeno_world_destroy(h)
                self._handle = ffi.NULL
        except Exception:  # interpreter teardown: cffi may already be gone
            pass

    # ---- dimensions ----
    num_envs = property(lambda self: self._num_envs)
    obs_dim = property(lambda self: self._obs_dim)
    action_dim = property(lambda self: self._action_dim)
    num_bodies = property(lambda self: self._num_bodies)
    num_joints = property(lambda self: self._num_joints)
    num_sensors = property(lambda self: self._num_sensors)
    num_geoms = property(lambda self: self._num_geoms)
    timestep = property(lambda self: self._timestep)
    memory_usage = property(lambda self: self._memory_usage)
    gpu_memory_usage = property(lambda self: self._gpu_memory_usage)
    max_contacts_per_env = property(lambda self: self._max_contacts_per_env)

    @property
    def handle(self):
        return self._handle

    def _view(self, ptr, shape, dtype=np.float32, cache_key=None) -> np.ndarray:
        if ptr == ffi.NULL:
            return np.zeros(shape, dtype=dtype)
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        arr = np.frombuffer(ffi.buffer(ptr, n), dtype=dtype).reshape(shape)
        if cache_key is not None:
            self._cached_arrays[cache_key] = ZeroCopyArray(arr, self, ptr)
        return arr

    # ---- stepping (reference _ffi.py:622-700) ----
    def step(self, actions: np.ndarray, substeps: int = 0) -> None:
        a = np.ascontiguousarray(actions, dtype=np.float32).ravel()
        _check(_lib.zeno_world_step(self._handle, _f32ptr(a), substeps), "Step")

    def step_subset(self, actions: np.ndarray, env_mask: np.ndarray, substeps: int = 0) -> None:
        a = np.ascontiguousarray(actions, dtype=np.float32).ravel()
        m = np.ascontiguousarray(env_mask, dtype=np.uint8)
        _check(_lib.zeno_world_step_subset(self._handle, _f32ptr(a), _u8ptr(m), substeps), "Step subset")

    def step_async(self, actions, substeps: int = 0) -> None:
        """Queue a step without synchronizing.  ``actions`` may be a host array or any
        object with ``__cuda_array_interface__`` / ``data_ptr()`` (device float32)."""
        if hasattr(actions, "data_ptr"):
            ptr = ffi.cast("float*", actions.data_ptr())
        elif hasattr(actions, "__cuda_array_interface__"):
            ptr = ffi.cast("float*", actions.__cuda_array_interface__["data"][0])
        else:
            actions = np.ascontiguousarray(actions, dtype=np.float32).ravel()
            ptr = _f32ptr(actions)
        _check(_lib.zeno_world_step_async(self._handle, ptr, substeps), "Step")

    def synchronize(self) -> None:
        _check(_lib.zeno_world_synchronize(self._handle), "Synchronize")

    def reset(self, mask: Optional[np.ndarray] = None) -> None:
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        _check(_lib.zeno_world_reset(self._handle, _u8ptr(m)), "Reset")

    def reset_to_state(self, positions, quaternions, velocities=None, angular_velocities=None, mask=None) -> None:
        cv = lambda x: None if x is None else np.ascontiguousarray(x, dtype=np.float32)
        p, q, v, w = cv(positions), cv(quaternions), cv(velocities), cv(angular_velocities)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        fp = lambda x: ffi.NULL if x is None else _f32ptr(x)
        _check(_lib.zeno_world_reset_to_state(self._handle, fp(p), fp(q), fp(v), fp(w), _u8ptr(m)), "Reset to state")

    # ---- zero-copy state (reference _ffi.py:765-1010) ----
    def _body4(self, fn, key, zero_copy):
        arr = self._view(fn(self._handle), (self._num_envs, self._num_bodies, 4), cache_key=key if zero_copy else None)
        return arr if zero_copy else arr.copy()

    def get_observations(self, zero_copy: bool = False) -> np.ndarray:
        arr = self._view(_lib.zeno_world_get_observations(self._handle), (self._num_envs, self._obs_dim),
                         cache_key="observations" if zero_copy else None)
        return arr if zero_copy else arr.copy()

    def get_rewards(self) -> np.ndarray:
        return self._view(_lib.zeno_world_get_rewards(self._handle), (self._num_envs,)).copy()

    def get_dones(self) -> np.ndarray:
        return self._view(_lib.zeno_world_get_dones(self._handle), (self._num_envs,), np.uint8).copy()

    def get_body_positions(self, zero_copy: bool = True):
        return self._body4(_lib.zeno_world_get_body_positions, "body_positions", zero_copy)

    def get_body_quaternions(self, zero_copy: bool = True):
        return self._body4(_lib.zeno_world_get_body_quaternions, "body_quaternions", zero_copy)

    def get_body_velocities(self, zero_copy: bool = True):
        return self._body4(_lib.zeno_world_get_body_velocities, "body_velocities", zero_copy)

    def get_body_angular_velocities(self, zero_copy: bool = True):
        return self._body4(_lib.zeno_world_get_body_angular_velocities, "body_angular_velocities", zero_copy)

    def get_body_accelerations(self, zero_copy: bool = True):
        return self._body4(_lib.zeno_world_get_body_accelerations, "body_accelerations", zero_copy)

    def _joint(self, fn, key, zero_copy):
        stride = max(self._num_joints, 1)
        arr = self._view(fn(self._handle), (self._num_envs, stride), cache_key=key if zero_copy else None)
        arr = arr[:, : self._num_joints]
        return arr if zero_copy else arr.copy()

    def get_joint_positions(self, zero_copy: bool = True):
        return self._joint(_lib.zeno_world_get_joint_positions, "joint_positions", zero_copy)

    def get_joint_velocities(self, zero_copy: bool = True):
        return self._joint(_lib.zeno_world_get_joint_velocities, "joint_velocities", zero_copy)

    def get_joint_forces(self, zero_copy: bool = True):
        return self._joint(_lib.zeno_world_get_joint_forces, "joint_forces", zero_copy)

    def get_contacts(self, zero_copy: bool = True) -> np.ndarray:
        arr = self._view(_lib.zeno_world_get_contacts(self._handle), (self._num_envs, self._max_contacts_per_env),
                         CONTACT_DTYPE, cache_key="contacts" if zero_copy else None)
        return arr if zero_copy else arr.copy()

    def get_contact_counts(self) -> np.ndarray:
        return self._view(_lib.zeno_world_get_contact_counts(self._handle), (self._num_envs,), np.uint32).copy()

    def get_sensor_data(self, zero_copy: bool = True) -> np.ndarray:
        arr = self._view(_lib.zeno_world_get_sensor_data(self._handle), (self._num_envs, self._obs_dim),
                         cache_key="sensor_data" if zero_copy else None)
        return arr if zero_copy else arr.copy()

    # ---- device views (extension) ----
    _DEVICE = {
        "observations": ("zeno_world_get_observations_device", lambda w: (w._num_envs, w._obs_dim), "<f4"),
        "rewards": ("zeno_world_get_rewards_device", lambda w: (w._num_envs,), "<f4"),
        "dones": ("zeno_world_get_dones_device", lambda w: (w._num_envs,), "|u1"),
        "body_positions": ("zeno_world_get_body_positions", lambda w: (w._num_envs, w._num_bodies, 4), "<f4"),
        "body_quaternions": ("zeno_world_get_body_quaternions", lambda w: (w._num_envs, w._num_bodies, 4), "<f4"),
        "body_velocities": ("zeno_world_get_body_velocities", lambda w: (w._num_envs, w._num_bodies, 4), "<f4"),
        "contact_counts": ("zeno_world_get_contact_counts", lambda w: (w._num_envs,), "<u4"),
        # 64-byte contact records viewed as 16 floats (position_pen, normal_friction, the
        # uint32 indices as raw bits, impulses)
        "contacts": ("zeno_world_get_contacts", lambda w: (w._num_envs, w._max_contacts_per_env, 16), "<f4"),
    }

    def device_array(self, name: str) -> CudaArray:
        fn, shape, ts = self._DEVICE[name]
        ptr = int(ffi.cast("uintptr_t", getattr(_lib, fn)(self._handle)))
        return CudaArray(ptr, shape(self), ts, self)

    # ---- mutation (reference _ffi.py:1012-1084) ----
    def set_body_positions(self, positions, mask=None) -> None:
        p = np.ascontiguousarray(positions, dtype=np.float32)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        _check(_lib.zeno_world_set_body_positions(self._handle, _f32ptr(p), _u8ptr(m)), "Set body positions")

    def set_body_velocities(self, velocities, mask=None) -> None:
        v = np.ascontiguousarray(velocities, dtype=np.float32)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        _check(_lib.zeno_world_set_body_velocities(self._handle, _f32ptr(v), _u8ptr(m)), "Set body velocities")

    def set_gravity(self, gravity: Tuple[float, float, float]) -> None:
        _check(_lib.zeno_world_set_gravity(self._handle, gravity[0], gravity[1], gravity[2]), "Set gravity")

    def set_timestep(self, timestep: float) -> None:
        _check(_lib.zeno_world_set_timestep(self._handle, timestep), "Set timestep")
        self._timestep = timestep

    # ---- extensions ----
    def set_task(self, enabled: bool = True, body: int = 1, z_min: float = -np.inf, z_max: float = np.inf,
                 auto_reset: bool = False, noise: float = 0.0, forward_weight: float = 1.0,
                 alive_bonus: float = 1.0, ctrl_cost: float = 0.01, seed: int = 0, env_offset: int = 0) -> None:
        t = ffi.new("ZenoTaskConfig*")
        t.enabled, t.body, t.auto_reset = int(enabled), body, int(auto_reset)
        t.z_min, t.z_max, t.noise = z_min, z_max, noise
        t.forward_weight, t.alive_bonus, t.ctrl_cost = forward_weight, alive_bonus, ctrl_cost
        t.seed, t.env_offset = seed, env_offset
        _check(_lib.zeno_world_set_task(self._handle, t), "Set task")

    def set_narrow_phase(self, mode: int) -> None:
        """0: the reference's GPU narrow phase (default); 1: its CPU collision routines
        (detectCollision: sphere/capsule/box/plane pairs, geoms placed by body pose); 2: as
        1, plus box-capsule pairs through its GJK + EPA."""
        _check(_lib.zeno_world_set_narrow_phase(self._handle, int(mode)), "Set narrow phase")

    def get_narrow_phase(self) -> int:
        return int(_lib.zeno_world_get_narrow_phase(self._handle))

    def set_broad_phase(self, mode: int) -> None:
        """0: auto (grid above 512 geoms); 1: all candidate pairs; 2: hashed grid.  Same
        slots either way."""
        _check(_lib.zeno_world_set_broad_phase(self._handle, int(mode)), "Set broad phase")

    def get_broad_phase(self) -> int:
        return int(_lib.zeno_world_get_broad_phase(self._handle))

    def set_launch(self, lanes: int, envs_per_block: int) -> None:
        _check(_lib.zeno_world_set_launch(self._handle, lanes, envs_per_block), "Set launch")

    def get_launch(self) -> Tuple[int, int]:
        l, e = ffi.new("int*"), ffi.new("int*")
        _lib.zeno_world_get_launch(self._handle, l, e)
        return l[0], e[0]

    def set_stream(self, cuda_stream: int) -> None:
        _check(_lib.zeno_world_set_stream(self._handle, ffi.cast("void*", cuda_stream)), "Set stream")

    @property
    def stream(self) -> int:
        return int(ffi.cast("uintptr_t", _lib.zeno_world_get_stream(self._handle)))

    @property
    def device(self) -> int:
        return _lib.zeno_world_device(self._handle)

    def model_table(self, name: str) -> bytes:
        n = ffi.new("uint64_t*")
        p = _lib.zeno_world_model_table(self._handle, name.encode(), n)
        if p == ffi.NULL:
            raise KeyError(name)
        return bytes(ffi.buffer(p, n[0]))

    # ---- profiling / checkpoint / info (reference _ffi.py:1086-1162) ----
    def get_profiling_data(self) -> Dict[str, Any]:
        d = ffi.new("ZenoProfilingData*")
        if _lib.zeno_world_get_profiling(self._handle, d) != 0:
            return {}
        return {"integrate_ms": d.integrate_ns / 1e6, "collision_broad_ms": d.collision_broad_ns / 1e6,
                "collision_narrow_ms": d.collision_narrow_ns / 1e6,
                "constraint_solve_ms": d.constraint_solve_ns / 1e6, "total_step_ms": d.total_step_ns / 1e6,
                "num_contacts": d.num_contacts, "num_active_constraints": d.num_active_constraints}

    STAGES = ("prologue", "actions", "integrate", "broad_phase", "sort", "narrow_phase", "schedule", "joints",
              "contacts", "velocities", "joint_states_sensors", "write_back", "task", "epilogue")

    def get_stage_profile(self) -> Dict[str, float]:
        """Per-stage device cycles of the last synchronous step, averaged over the kernel's
        blocks, plus the block span ("span_cycles"), "ns_per_cycle", the slowest block's
        span ("max_span_cycles") and each stage's largest per-block cycles ("max_<stage>")
        (a world created with enable_profiling=True, either kernel; {} otherwise)."""
        k = len(self.STAGES)
        n = 2 * k + 3
        out = ffi.new("double[]", n)
        got = _lib.zeno_world_get_stage_cycles(self._handle, out, n)
        if got < n:
            return {}
        d = {name: out[i] for i, name in enumerate(self.STAGES)}
        d["span_cycles"], d["ns_per_cycle"], d["max_span_cycles"] = out[k], out[k + 1], out[k + 2]
        d.update({"max_" + name: out[k + 3 + i] for i, name in enumerate(self.STAGES)})
        return d

    def reset_profiling(self) -> None:
        _lib.zeno_world_reset_profiling(self._handle)

    def get_state(self) -> Dict[str, np.ndarray]:
        return {"body_positions": self.get_body_positions(zero_copy=False),
                "body_quaternions": self.get_body_quaternions(zero_copy=False),
                "body_velocities": self.get_body_velocities(zero_copy=False),
                "body_angular_velocities": self.get_body_angular_velocities(zero_copy=False),
                "joint_positions": self.get_joint_positions(zero_copy=False),
                "joint_velocities": self.get_joint_velocities(zero_copy=False)}

    def set_state(self, state: Dict[str, np.ndarray]) -> None:
        self.reset_to_state(positions=state["body_positions"], quaternions=state["body_quaternions"],
                            velocities=state.get("body_velocities"),
                            angular_velocities=state.get("body_angular_velocities"))

    def get_info(self) -> Dict[str, Any]:
        i = ffi.new("ZenoInfo*")
        _lib.zeno_world_get_info(self._handle, i)
        return {"num_envs": i.num_envs, "num_bodies": i.num_bodies, "num_joints": i.num_joints,
                "num_actuators": i.num_actuators, "num_sensors": i.num_sensors, "num_geoms": i.num_geoms,
                "obs_dim": i.obs_dim, "action_dim": i.action_dim, "timestep": i.timestep,
                "memory_usage_mb": i.memory_usage / (1024 * 1024),
                "gpu_memory_usage_mb": i.gpu_memory_usage / (1024 * 1024),
                "metal_available": bool(i.metal_available)}
