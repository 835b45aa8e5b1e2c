"""Shared helpers for the parity tests: the same world is created twice, once on the
GPU through the C ABI (zeno_b200.ZenoWorld) and once in the CPU oracle, driven with
the same seeded actions, and every ABI-visible buffer is compared bit for bit."""
from __future__ import annotations

import numpy as np

from oracle.zeno_oracle import OracleWorld
from zeno_b200 import ZenoWorld, scenes

# (scene, substeps, contact_iterations, max_contacts, action scale)
CONFIGS = {
    "pendulum": dict(xml=scenes.pendulum, substeps=4, iters=4, max_contacts=64, act=1.0),
    "cartpole": dict(xml=scenes.cartpole, substeps=1, iters=4, max_contacts=64, act=1.0),
    "ant": dict(xml=scenes.ant, substeps=4, iters=4, max_contacts=64, act=1.0),
    "humanoid": dict(xml=scenes.humanoid, substeps=4, iters=4, max_contacts=64, act=0.4, timestep=0.015),
    "pendulum_asset": dict(xml=scenes.pendulum_asset, substeps=1, iters=4, max_contacts=64, act=5.0),
}

FIELDS = ["positions", "quaternions", "velocities", "angular_velocities", "accelerations", "joint_positions",
          "joint_velocities", "joint_torques", "observations", "rewards", "dones", "contacts", "contact_counts"]


def make_pair(name: str, num_envs: int, semantics: str = "reference", **over):
    c = dict(CONFIGS[name])
    c.update(over)
    xml = c["xml"]() if callable(c["xml"]) else c["xml"]
    kw = dict(num_envs=num_envs, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
              max_contacts_per_env=c["max_contacts"], substeps=c["substeps"], semantics=semantics)
    return ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw), c


def product_state(w: ZenoWorld) -> dict:
    return {
        "positions": w.get_body_positions(zero_copy=False),
        "quaternions": w.get_body_quaternions(zero_copy=False),
        "velocities": w.get_body_velocities(zero_copy=False),
        "angular_velocities": w.get_body_angular_velocities(zero_copy=False),
        "accelerations": w.get_body_accelerations(zero_copy=False),
        "joint_positions": w.get_joint_positions(zero_copy=False),
        "joint_velocities": w.get_joint_velocities(zero_copy=False),
        "joint_torques": w.get_joint_forces(zero_copy=False),
        "observations": w.get_observations(zero_copy=False),
        "rewards": w.get_rewards(),
        "dones": w.get_dones(),
        "contacts": w.get_contacts(zero_copy=False),
        "contact_counts": w.get_contact_counts(),
    }


def bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    return a.view(np.uint8)


def diff_report(p: dict, o: dict, fields=FIELDS) -> list:
    """Fields whose bytes differ, with the first differing env."""
    bad = []
    for f in fields:
        pa, oa = np.ascontiguousarray(p[f]), np.ascontiguousarray(o[f])
        if pa.shape != oa.shape:
            bad.append(f"{f}: shape {pa.shape} vs {oa.shape}")
            continue
        pb, ob = bits(pa).reshape(pa.shape[0], -1), bits(oa).reshape(oa.shape[0], -1)
        rows = np.nonzero((pb != ob).any(axis=1))[0]
        if rows.size:
            bad.append(f"{f}: {rows.size} envs differ, first env {rows[0]}")
    return bad


def actions(rng: np.random.Generator, nsteps: int, num_envs: int, act_dim: int, scale: float) -> np.ndarray:
    return rng.uniform(-scale, scale, size=(nsteps, num_envs, act_dim)).astype(np.float32)
