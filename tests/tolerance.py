"""Helpers for the tolerance checks against the oracle's literal arithmetic.

The literal arithmetic (oracle/oracle_literal.cpp) restates the reference's Metal kernels
expression by expression in plain IEEE single precision; the "contracted" arithmetic is the
same source compiled with FMA contraction.  The product evaluates the oracle's canonical
arithmetic bit for bit, so these checks measure how far that canonical arithmetic lies from
the reference's own.

Error measure (stated once, used by every tolerance test): for a field f (positions,
quaternions, linear velocities, angular velocities, joint positions, joint velocities), the
normwise relative error over a batch of environments is

    err(f) = max_i |f_test[i] - f_ref[i]| / max_i |f_ref[i]|

over every component i of every environment (xyz only for float4 body arrays).  Per
environment, the same quotient over that environment's components.
"""
from __future__ import annotations

import numpy as np

from oracle.zeno_oracle import OracleWorld
from parity import CONFIGS
from zeno_b200.initial_state import _rot, joint_noise_state

BODY4 = ("positions", "velocities", "angular_velocities")
FIELDS = ("positions", "quaternions", "velocities", "angular_velocities", "joint_positions", "joint_velocities")


def comp(state: dict, f: str) -> np.ndarray:
    a = state[f]
    return a[..., :3] if f in BODY4 else a


def batch_err(test: dict, ref: dict, f: str) -> float:
    a, b = comp(test, f).astype(np.float64), comp(ref, f).astype(np.float64)
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / den) if den > 0 else float(np.abs(a - b).max())


def env_err(test: dict, ref: dict, f: str) -> np.ndarray:
    a, b = comp(test, f).astype(np.float64), comp(ref, f).astype(np.float64)
    E = a.shape[0]
    num = np.abs(a - b).reshape(E, -1).max(1)
    den = np.abs(b).reshape(E, -1).max(1)
    return num / np.maximum(den, np.finfo(np.float64).tiny)


def oracle(name: str, num_envs: int, arithmetic: str, **over) -> tuple:
    c = dict(CONFIGS[name])
    c.update(over)
    xml = c["xml"]() if callable(c["xml"]) else c["xml"]
    w = OracleWorld(xml, num_envs=num_envs, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
                    max_contacts_per_env=c["max_contacts"], substeps=c["substeps"], arithmetic=arithmetic)
    return w, c, xml


# ---- initial states: joint-coordinate noise applied by forward kinematics -------------

def noisy_initial_state(w: OracleWorld, rng: np.random.Generator, qpos: float, qvel: float = 0.0,
                        num_envs: int = 0) -> dict:
    """Environment 0's initial pose with joint-coordinate noise (zeno_b200.initial_state:
    hinge / slider coordinates U(-qpos, qpos), free joints' six coordinates U(-qpos, qpos),
    joint rates U(-qvel, qvel)) for num_envs environments (default: the world's)."""
    s = w.state()
    return joint_noise_state(w.model_table("bodies"), w.model_table("joints"), s["positions"][0],
                             s["quaternions"][0], num_envs or w.num_envs, rng, qpos, qvel)


def apply_state(world, st: dict) -> None:
    world.reset_to_state(st["positions"], st["quaternions"], st["velocities"], st["angular_velocities"])


# ---- 1000-step statistics --------------------------------------------------------------

def energy(state: dict, inv_mass_inertia: np.ndarray, g: float = 9.81) -> np.ndarray:
    """Per-environment energy sum over dynamic bodies of 1/2 m v.v + 1/2 w_b^T I w_b + m g z
    (w_b: angular velocity in the body frame, I: the body's diagonal inertia, z: the height
    of the body origin), in float64."""
    imi = inv_mass_inertia.astype(np.float64)
    dyn = imi[..., 0] > 1e-8
    m = np.where(dyn, 1.0 / np.where(dyn, imi[..., 0], 1.0), 0.0)
    inv_i = imi[..., 1:]
    I = np.where(inv_i > 0, 1.0 / np.where(inv_i > 0, inv_i, 1.0), 0.0)
    v = state["velocities"][..., :3].astype(np.float64)
    q = state["quaternions"].astype(np.float64)
    w = state["angular_velocities"][..., :3].astype(np.float64)
    wb = _rot(q * np.array([-1.0, -1.0, -1.0, 1.0]), w)
    z = state["positions"][..., 2].astype(np.float64)
    e = 0.5 * m * (v * v).sum(-1) + 0.5 * (I * wb * wb).sum(-1) + m * g * z
    return (e * dyn).sum(-1)


def valid_contacts(contacts: np.ndarray, counts: np.ndarray, max_contacts: int) -> np.ndarray:
    """Per environment: slots of the live list (index < min(count, M)) holding a contact
    (penetration >= 0)."""
    n = np.minimum(counts.astype(np.int64), max_contacts)
    live = np.arange(max_contacts)[None, :] < n[:, None]
    return ((contacts["position_pen"][..., 3] >= 0) & live).sum(1)


def slog(x: np.ndarray) -> np.ndarray:
    """sign(x) log10(1 + |x|): the reference Humanoid's energy drift spans 30 orders of
    magnitude across environments (some explode), so means are compared on this scale."""
    return np.sign(x) * np.log10(1.0 + np.abs(x))


def ks_pvalue(x: np.ndarray, y: np.ndarray) -> float:
    """Two-sample Kolmogorov-Smirnov p-value (distributions equal)."""
    if np.array_equal(np.sort(x), np.sort(y)):
        return 1.0
    from scipy.stats import ks_2samp
    return float(ks_2samp(x, y).pvalue)


def two_sample_z(x: np.ndarray, y: np.ndarray) -> float:
    """(mean x - mean y) over its standard error."""
    se = np.sqrt(x.var(ddof=1) / x.size + y.var(ddof=1) / y.size)
    d = x.mean() - y.mean()
    return float(d / se) if se > 0 else (0.0 if d == 0 else float("inf"))
