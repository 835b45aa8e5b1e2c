"""The sm_100a step, through the C ABI, against the reference's own arithmetic.

The bit-exact parity tests compare the product with the oracle's canonical arithmetic,
which was designed together with the kernel.  These tests instead compare it with the
oracle's LITERAL arithmetic (oracle/oracle_literal.cpp: the reference's Metal kernels
statement by statement in plain IEEE single precision), and use the same source compiled
with FMA contraction ("contracted") as the yardstick of what two legitimate builds of the
reference's own source disagree by.  Error measure and initial states: tests/tolerance.py.

* Pendulum (1024 envs) and Cartpole (4096 envs), BASELINE.json configs 1 and 2 with their
  initial noise: positions, quaternions and linear velocities within north_star's 1e-5
  (after 1 step) and 1e-3 (after 10 steps) normwise relative error; angular velocities and
  joint rates (derived from a quaternion change over one substep, a cancellation that costs
  every arithmetic about three digits) within the larger of that tolerance and 4x the
  literal/contracted spread; contact counts and pair lists identical.
* Ant (16384-env world, 512 sampled envs) and Humanoid (4096-env world, 256 sampled envs):
  chaotic at the rounding level in the reference's own arithmetic (test_literal_oracle.py),
  so the product is held to the literal/contracted spread: median and 90th percentile of
  the per-environment error within 4x of that spread, after 1 and 10 steps.
* 1000-step statistics for all four, 1024 envs: per-environment energy drift and mean
  valid-contact count, product against literal: two-sample comparison of means (|z| <= 4;
  the drift on a signed log scale, since some reference Humanoids explode) and of
  distributions (Kolmogorov-Smirnov p >= 1e-3).
"""
import numpy as np
import pytest

from parity import CONFIGS, actions, product_state
from tolerance import (FIELDS, apply_state, batch_err, energy, env_err, ks_pvalue, noisy_initial_state, oracle,
                       slog, two_sample_z)
from zeno_b200 import ZenoWorld

pytestmark = pytest.mark.gpu

EXACT = ("positions", "quaternions", "velocities")
RATE = ("angular_velocities", "joint_positions", "joint_velocities")
NOISE = {"pendulum": (0.1, 0.0), "cartpole": (0.01, 0.01), "ant": (0.1, 0.0), "humanoid": (0.01, 0.0)}


def _gpu_world(name, E):
    c = CONFIGS[name]
    xml = c["xml"]() if callable(c["xml"]) else c["xml"]
    return ZenoWorld(mjcf_string=xml, num_envs=E, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
                     max_contacts_per_env=c["max_contacts"], substeps=c["substeps"])


def _setup(name, E_gpu, sample, seed=0):
    """GPU world of E_gpu envs and literal/contracted oracles of the sampled envs, all from
    the same noisy initial state; returns them with the per-step actions."""
    qpos, qvel = NOISE[name]
    g = _gpu_world(name, E_gpu)
    probe, c, _ = oracle(name, 1, "literal")
    st = noisy_initial_state(probe, np.random.default_rng(seed), qpos, qvel, num_envs=E_gpu)
    apply_state(g, st)
    sub = {k: v[sample] for k, v in st.items()}
    refs = {}
    for a in ("literal", "contracted"):
        refs[a] = oracle(name, len(sample), a)[0]
        apply_state(refs[a], sub)
    acts = actions(np.random.default_rng(seed + 1), 10, E_gpu, max(g.action_dim, 1), c["act"])
    return g, refs, acts


def _sampled(state, sample):
    return {k: (v[sample] if isinstance(v, np.ndarray) and v.ndim >= 1 and v.shape[0] > max(sample) else v)
            for k, v in state.items()}


@pytest.mark.parametrize("name,E", [("pendulum", 1024), ("cartpole", 4096)])
def test_within_tolerance_well_conditioned(name, E):
    sample = np.arange(E)
    g, refs, acts = _setup(name, E, sample)
    for k in range(10):
        g.step(acts[k])
        for r in refs.values():
            r.step(acts[k][sample])
        if k + 1 not in (1, 10):
            continue
        tol = 1e-5 if k == 0 else 1e-3
        p, lit, con = product_state(g), refs["literal"].state(), refs["contracted"].state()
        for f in EXACT:
            e = batch_err(p, lit, f)
            assert e <= tol, f"{name} step {k + 1} {f}: {e:.3g} > {tol}"
        for f in RATE:
            e, spread = batch_err(p, lit, f), batch_err(con, lit, f)
            assert e <= max(tol, 4.0 * spread), f"{name} step {k + 1} {f}: {e:.3g} (spread {spread:.3g})"
        assert np.array_equal(p["contact_counts"], lit["contact_counts"])
        n_live = min(int(lit["contact_counts"].max()), g.max_contacts_per_env)
        assert np.array_equal(p["contacts"]["indices"][:, :n_live], lit["contacts"]["indices"][:, :n_live])


@pytest.mark.parametrize("name,E,n", [("ant", 16384, 512), ("humanoid", 4096, 256)])
def test_within_reference_spread_chaotic(name, E, n):
    sample = np.sort(np.random.default_rng(3).choice(E, size=n, replace=False))
    g, refs, acts = _setup(name, E, sample)
    for k in range(10):
        g.step(acts[k])
        for r in refs.values():
            r.step(acts[k][sample])
        if k + 1 not in (1, 10):
            continue
        p = _sampled(product_state(g), sample)
        lit, con = refs["literal"].state(), refs["contracted"].state()
        for f in FIELDS[:4]:
            ep, ec = env_err(p, lit, f), env_err(con, lit, f)
            for q in (0.5, 0.9):
                a, b = np.quantile(ep, q), np.quantile(ec, q)
                assert a <= 4.0 * b, f"{name} step {k + 1} {f} q{q}: product {a:.3g} vs contracted {b:.3g}"


@pytest.mark.parametrize("name", ["pendulum", "cartpole", "ant", "humanoid"])
def test_1000_step_statistics(name):
    import torch
    E, N = 1024, 1000
    sample = np.arange(E)
    g, refs, _ = _setup(name, E, sample)
    lit = refs["literal"]
    c = CONFIGS[name]
    M = g.max_contacts_per_env
    imi = lit.raw("inv_mass_inertia").reshape(E, lit.num_bodies, 4)
    e0 = energy(product_state(g), imi)
    e0_lit = energy(lit.state(), imi)
    assert np.array_equal(e0, e0_lit)
    rng = np.random.default_rng(99)
    con_d = torch.as_tensor(g.device_array("contacts"), device="cuda")
    cnt_d = torch.as_tensor(g.device_array("contact_counts"), device="cuda")
    slot = torch.arange(M, device="cuda")[None, :]
    vc_gpu = torch.zeros(E, dtype=torch.float64, device="cuda")
    vc_lit = np.zeros(E)
    import os
    threads = max(1, min(32, os.cpu_count() or 1))
    for k in range(N):
        a = actions(rng, 1, E, max(g.action_dim, 1), c["act"])
        g.step(a[0])
        live = slot < torch.clamp(cnt_d.to(torch.int64), max=M)[:, None]
        vc_gpu += ((con_d[:, :, 3] >= 0) & live).sum(1).to(torch.float64)
        lit.run(a, threads=threads)
        s = lit.state()
        n_live = np.minimum(s["contact_counts"].astype(np.int64), M)
        vc_lit += ((s["contacts"]["position_pen"][..., 3] >= 0) & (np.arange(M)[None] < n_live[:, None])).sum(1)
    vc_gpu = vc_gpu.cpu().numpy() / N
    vc_lit /= N
    d_gpu = energy(product_state(g), imi) - e0
    d_lit = energy(lit.state(), imi) - e0
    z_e, z_c = two_sample_z(slog(d_gpu), slog(d_lit)), two_sample_z(vc_gpu, vc_lit)
    p_e, p_c = ks_pvalue(d_gpu, d_lit), ks_pvalue(vc_gpu, vc_lit)
    print(f"{name}: energy drift median product {np.median(d_gpu):.6g} literal {np.median(d_lit):.6g}, "
          f"mean slog product {slog(d_gpu).mean():.4f} literal {slog(d_lit).mean():.4f} z {z_e:.2f} KS p {p_e:.3g}; "
          f"valid contacts per step product {vc_gpu.mean():.6g} literal {vc_lit.mean():.6g} z {z_c:.2f} KS p {p_c:.3g}")
    assert np.isfinite(slog(d_gpu)).all() and np.isfinite(slog(d_lit)).all()
    assert abs(z_e) <= 4.0 and p_e >= 1e-3, f"{name}: energy drift z = {z_e:.2f}, KS p = {p_e:.3g}"
    assert abs(z_c) <= 4.0 and p_c >= 1e-3, f"{name}: valid-contact z = {z_c:.2f}, KS p = {p_c:.3g}"
