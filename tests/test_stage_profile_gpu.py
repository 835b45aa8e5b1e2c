"""Stage profile of a profiling world (ZenoConfig.enable_profiling; the reference fills
ZenoProfilingData's stage fields, src/world/world.zig:1021-1216, main.zig:666-683).

The instrumented kernel instantiation must step exactly like the default one, and fill the
stage fields and zeno_world_get_stage_cycles."""
import numpy as np
import pytest

from parity import CONFIGS, actions, diff_report, product_state
from zeno_b200 import ZenoWorld

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["ant", "humanoid"])
def test_profiling_world_bit_identical_and_filled(name):
    c = CONFIGS[name]
    kw = dict(mjcf_string=c["xml"](), num_envs=64, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
              max_contacts_per_env=c["max_contacts"], substeps=c["substeps"])
    w0 = ZenoWorld(**kw)
    w1 = ZenoWorld(enable_profiling=True, **kw)
    assert w1.get_stage_profile() == {}  # no step yet
    acts = actions(np.random.default_rng(3), 5, 64, w0.action_dim, c["act"])
    for s in range(5):
        w0.step(acts[s])
        w1.step(acts[s])
    assert not diff_report(product_state(w1), product_state(w0))
    prof = w1.get_stage_profile()
    stages = ZenoWorld.STAGES
    assert all(prof[k] >= 0 for k in stages)
    for k in ("integrate", "broad_phase", "narrow_phase", "joints", "contacts", "velocities"):
        assert prof[k] > 0, k
    assert prof["span_cycles"] >= 0.9 * sum(prof[k] for k in stages)
    assert 0.2 < prof["ns_per_cycle"] < 5.0
    assert prof["max_span_cycles"] >= prof["span_cycles"]
    assert all(prof["max_" + k] >= prof[k] for k in stages)
    d = w1.get_profiling_data()
    for k in ("integrate_ms", "collision_broad_ms", "collision_narrow_ms", "constraint_solve_ms", "total_step_ms"):
        assert d[k] > 0, k
    assert d["constraint_solve_ms"] < d["total_step_ms"]
    assert w0.get_stage_profile() == {}
    assert w0.get_profiling_data()["integrate_ms"] == 0.0


@pytest.mark.parametrize("name,lanes,epb,mode", [("ant", 8, 4, 0), ("humanoid", 8, 4, 1), ("humanoid", 32, 1, 2)])
def test_general_kernel_profile_bit_identical_and_filled(name, lanes, epb, mode):
    """The general kernel's stage-profiling instantiation (forced launch shape, or a narrow
    phase the compressed-state kernel does not run) steps exactly like the default one."""
    c = CONFIGS[name]
    kw = dict(mjcf_string=c["xml"](), num_envs=16, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
              max_contacts_per_env=c["max_contacts"], substeps=c["substeps"])
    w0 = ZenoWorld(**kw)
    w1 = ZenoWorld(enable_profiling=True, **kw)
    for w in (w0, w1):
        w.set_narrow_phase(mode)
        w.set_launch(lanes, epb)
    acts = actions(np.random.default_rng(5), 4, 16, w0.action_dim, c["act"])
    for s in range(4):
        w0.step(acts[s])
        w1.step(acts[s])
    assert not diff_report(product_state(w1), product_state(w0))
    prof = w1.get_stage_profile()
    for k in ("prologue", "integrate", "broad_phase", "narrow_phase", "joints", "contacts", "velocities", "epilogue"):
        assert prof[k] > 0, k
    assert prof["span_cycles"] >= 0.9 * sum(prof[k] for k in ZenoWorld.STAGES)
    assert prof["max_span_cycles"] >= prof["span_cycles"]
    assert w1.get_profiling_data()["constraint_solve_ms"] > 0
