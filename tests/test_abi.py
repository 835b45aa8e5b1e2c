"""The C-ABI boundary: libzeno.so loads without a GPU, exports every function declared in
include/zeno.h (the reference's 54 exports plus the extensions), keeps the reference's
struct sizes, and follows its NULL-handle error conventions (src/main.zig)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "zeno.h"
LIB = ROOT / "zeno_b200" / "lib" / "libzeno.so"
REF_SYMBOLS = ROOT / "tests" / "golden" / "reference_abi_symbols.txt"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(zeno_[A-Za-z0-9_]+)\s*\(", text)))


def exported():
    out = subprocess.check_output(["nm", "-D", "--defined-only", str(LIB)], text=True)
    return {ln.split()[-1] for ln in out.splitlines() if ln.split() and ln.split()[-1].startswith("zeno_")}


def test_header_functions_exported():
    missing = [n for n in declared() if n not in exported()]
    assert not missing, missing


def test_reference_abi_exported():
    ref = [s.strip() for s in REF_SYMBOLS.read_text().split() if s.strip()]
    assert len(ref) == 54
    missing = [n for n in ref if n not in exported()]
    assert not missing, missing
    assert set(ref) <= set(declared())


class ZenoConfig(ctypes.Structure):
    _fields_ = [("num_envs", ctypes.c_uint32), ("timestep", ctypes.c_float), ("contact_iterations", ctypes.c_uint32),
                ("max_contacts_per_env", ctypes.c_uint32), ("seed", ctypes.c_uint64), ("substeps", ctypes.c_uint32),
                ("enable_profiling", ctypes.c_bool), ("max_bodies_per_env", ctypes.c_uint32),
                ("max_joints_per_env", ctypes.c_uint32), ("max_geoms_per_env", ctypes.c_uint32)]


class ZenoInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("num_envs", "num_bodies", "num_joints", "num_actuators", "num_sensors",
                                               "num_geoms", "obs_dim", "action_dim")] + \
               [("timestep", ctypes.c_float), ("memory_usage", ctypes.c_uint64), ("gpu_memory_usage", ctypes.c_uint64),
                ("metal_available", ctypes.c_bool)]


def test_struct_layouts_match_reference():
    # extern structs of src/main.zig:75-113 under the C ABI
    assert ctypes.sizeof(ZenoConfig) == 48
    assert ctypes.sizeof(ZenoInfo) == 64


@pytest.fixture(scope="module")
def L():
    lib = ctypes.CDLL(str(LIB))
    lib.zeno_version.restype = ctypes.c_char_p
    lib.zeno_error_string.restype = ctypes.c_char_p
    lib.zeno_metal_available.restype = ctypes.c_bool
    for f in ("zeno_world_get_observations", "zeno_world_get_contacts", "zeno_world_get_body_positions",
              "zeno_swarm_create", "zeno_swarm_get_agent_states"):
        getattr(lib, f).restype = ctypes.c_void_p
    return lib


def test_version_and_errors(L):
    assert L.zeno_version() == b"0.1.0"
    assert L.zeno_error_string(0) == b"success"
    assert L.zeno_error_string(-4) == b"metal error"
    assert L.zeno_error_string(-6) == b"invalid argument"
    assert L.zeno_error_string(123) == b"unknown error"
    assert isinstance(L.zeno_metal_available(), bool)


def test_null_handle_conventions(L):
    assert L.zeno_world_step(None, None, 0) == -1
    assert L.zeno_world_step_subset(None, None, None, 0) == -1
    assert L.zeno_world_reset(None, None) == -1
    assert L.zeno_world_set_gravity(None, ctypes.c_float(0), ctypes.c_float(0), ctypes.c_float(0)) == -1
    assert L.zeno_world_set_timestep(None, ctypes.c_float(0.01)) == -1
    assert L.zeno_world_get_info(None, None) == -1
    assert L.zeno_world_get_observations(None) is None
    assert L.zeno_world_get_contacts(None) is None
    assert L.zeno_world_num_envs(None) == 0
    L.zeno_world_destroy(None)
    L.zeno_world_compact_memory(None)
    assert L.zeno_swarm_create(None, None) is None
    assert L.zeno_swarm_step(None, None, None) == -1
    assert L.zeno_swarm_get_agent_states(None) is None


def test_create_without_gpu_fails_cleanly(L):
    if L.zeno_metal_available():
        pytest.skip("a CUDA device is present")
    cfg = ZenoConfig(1, 0.0, 4, 64, 42, 1, False, 0, 0, 0)
    L.zeno_world_create_from_string.restype = ctypes.c_void_p
    h = L.zeno_world_create_from_string(b"<mujoco><worldbody/></mujoco>", ctypes.byref(cfg))
    assert h is None


def test_missing_file_returns_null(L):
    cfg = ZenoConfig(1, 0.0, 4, 64, 42, 1, False, 0, 0, 0)
    L.zeno_world_create.restype = ctypes.c_void_p
    assert L.zeno_world_create(b"/nonexistent/model.xml", ctypes.byref(cfg)) is None


def test_missing_library_fails_loudly_but_build_imports():
    """Without libzeno.so the package has no fallback: every library-backed name raises
    ImportError, while the build module and the pure-Python scenes still import (a fresh
    checkout must be able to run `python -m zeno_b200.build`)."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    code = (
        "import zeno_b200, zeno_b200.build, zeno_b200.scenes\n"
        "try:\n"
        "    from zeno_b200 import ZenoWorld\n"
        "except ImportError as e:\n"
        "    assert 'libzeno.so not found' in str(e), e\n"
        "    print('loud')\n"
    )
    env = dict(__import__("os").environ, ZENO_B200_LIB=str(root / "no_such_dir" / "libzeno.so"))
    out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "loud"
