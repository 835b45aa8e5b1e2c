"""The oracle's literal arithmetic (oracle/oracle_literal.cpp) against its canonical
arithmetic, on the CPU.

The canonical arithmetic is what the product kernel evaluates bit for bit (the GPU parity
tests hold it to that); the literal arithmetic restates the reference's Metal kernels
expression by expression in plain IEEE single precision; "contracted" is the literal source
compiled with FMA contraction, one of the rewrites the Metal compiler's default fast-math
build of the reference makes.  Error measure: tests/tolerance.py.

What these establish:
* on the well-conditioned BASELINE models (Pendulum, Cartpole) the canonical arithmetic meets
  north_star's tolerances against the literal one (1e-5 after 1 step, 1e-3 after 10) for
  positions, quaternions and linear velocities, with identical contact pair lists and counts;
  angular velocities and joint rates, which the reference derives from a quaternion change
  over one substep (all_shaders.metal:1948-1958, 1616-1620), lose about three digits to
  that cancellation in every arithmetic, and are held to the spread of the reference's own
  source under its two compilations;
* the reference Ant and Humanoid are chaotic at the rounding level: one unit in the last
  place of one coordinate, stepped in the literal arithmetic itself, moves the state by
  more than 1e-3 (relative) within one step.  No single-precision implementation can hold
  them to 1e-5; the canonical arithmetic stays within the literal/contracted spread.
"""
import numpy as np
import pytest

from parity import actions
from tolerance import (FIELDS, apply_state, batch_err, env_err, noisy_initial_state, oracle)

# BASELINE.json configs 1 and 2: initial noise (qpos, qvel) and the action scale
WELL = {"pendulum": (0.1, 0.0), "cartpole": (0.01, 0.01)}
EXACT = ("positions", "quaternions", "velocities")
RATE = ("angular_velocities", "joint_positions", "joint_velocities")


def _run(name, E, arithmetics, nsteps, seed=0, qpos=0.1, qvel=0.0):
    worlds = {a: oracle(name, E, a)[0] for a in arithmetics}
    c = oracle(name, 1, "canonical")[1]
    ref = next(iter(worlds.values()))
    st = noisy_initial_state(ref, np.random.default_rng(seed), qpos, qvel)
    for w in worlds.values():
        apply_state(w, st)
    acts = actions(np.random.default_rng(seed + 1), nsteps, E, max(ref.num_actuators, 1), c["act"])
    out = {}
    for k in range(nsteps):
        for w in worlds.values():
            w.step(acts[k])
        if k + 1 in (1, 10):
            out[k + 1] = {a: w.state() for a, w in worlds.items()}
    return out


def test_literal_known_answer_free_fall():
    """A free body under gravity, one substep, no contact (the sphere is 5 m up): the
    literal integrate (all_shaders.metal:394-462) is v = (v + (F m^-1) dt) 0.999,
    x = x + v dt, each operation rounded once, with F = g (1 / m^-1) from compute_forces,
    and xpbd_update_velocities (:1922-1961) then sets v = (x - x_prev) (1 / dt)."""
    xml = """<mujoco><option timestep="0.01"/><worldbody>
      <body name="b" pos="0 0 5"><joint type="free"/><geom type="sphere" size="0.1" mass="2"/></body>
      </worldbody></mujoco>"""
    from oracle.zeno_oracle import OracleWorld
    w = OracleWorld(xml, num_envs=1, substeps=1, arithmetic="literal")
    inv_m = np.float32(w.raw("inv_mass_inertia").reshape(1, -1, 4)[0, 1, 0])
    w.step(np.zeros((1, 1), np.float32))
    f32 = np.float32
    dt = f32(0.01)
    F = f32(-9.81) * (f32(1.0) / inv_m)
    v = (f32(0.0) + (F * inv_m) * dt) * f32(0.999)
    z = f32(5.0) + v * dt
    s = w.state()
    assert s["positions"][0, 1, 2] == z
    assert s["velocities"][0, 1, 2] == (z - f32(5.0)) * (f32(1.0) / dt)


@pytest.mark.parametrize("name", list(WELL))
def test_canonical_within_tolerance_well_conditioned(name):
    qpos, qvel = WELL[name]
    E = 256
    out = _run(name, E, ("canonical", "literal", "contracted"), 10, qpos=qpos, qvel=qvel)
    for n, tol in ((1, 1e-5), (10, 1e-3)):
        s = out[n]
        for f in EXACT:
            e = batch_err(s["canonical"], s["literal"], f)
            assert e <= tol, f"{name} step {n} {f}: {e:.3g} > {tol}"
        for f in RATE:
            e = batch_err(s["canonical"], s["literal"], f)
            spread = batch_err(s["contracted"], s["literal"], f)
            assert e <= max(tol, 4.0 * spread), f"{name} step {n} {f}: {e:.3g} (spread {spread:.3g})"
        for f in ("contact_counts",):
            assert np.array_equal(s["canonical"][f], s["literal"][f])
        n_live = min(int(s["literal"]["contact_counts"].max()), 64)
        assert np.array_equal(s["canonical"]["contacts"]["indices"][:, :n_live],
                              s["literal"]["contacts"]["indices"][:, :n_live])


@pytest.mark.parametrize("name", ["ant", "humanoid"])
def test_reference_models_chaotic_at_rounding_level(name):
    """One ulp of one coordinate, in the literal arithmetic, already exceeds the 1e-5
    tolerance after one step and the 1e-3 tolerance after ten (median over environments),
    so the tolerances cannot apply to these models; the canonical arithmetic's distance from
    the literal one is of the same size as the literal source's own distance under FMA
    contraction."""
    E = 128
    qpos = 0.1 if name == "ant" else 0.01
    worlds = _run(name, E, ("canonical", "literal", "contracted"), 1, qpos=qpos)[1]
    # the literal arithmetic against itself, one input perturbed by one ulp
    w0, c, _ = oracle(name, E, "literal")
    w1 = oracle(name, E, "literal")[0]
    st = noisy_initial_state(w0, np.random.default_rng(0), qpos)
    apply_state(w0, st)
    st1 = {k: v.copy() for k, v in st.items()}
    st1["positions"][:, 1, 2] = np.nextafter(st1["positions"][:, 1, 2], np.float32(np.inf))
    apply_state(w1, st1)
    acts = actions(np.random.default_rng(1), 10, E, max(w0.num_actuators, 1), c["act"])
    for k, tol in enumerate([1e-5] + [None] * 8 + [1e-3]):
        w0.step(acts[k])
        w1.step(acts[k])
        if tol is not None:
            sens = np.median(env_err(w1.state(), w0.state(), "positions"))
            assert sens > tol, f"{name} step {k + 1}: one-ulp sensitivity {sens:.3g}"
    for f in FIELDS[:4]:
        d_can = np.median(env_err(worlds["canonical"], worlds["literal"], f))
        d_con = np.median(env_err(worlds["contracted"], worlds["literal"], f))
        assert d_can <= 4.0 * d_con, f"{name} {f}: canonical {d_can:.3g} vs contracted {d_con:.3g}"


def test_literal_refused_for_corrected_semantics():
    from oracle.zeno_oracle import OracleWorld
    from zeno_b200 import scenes
    w = OracleWorld(scenes.ant(), num_envs=1, semantics="corrected")
    assert w.set_arithmetic("literal") != 0
    assert w.set_arithmetic("canonical") == 0
