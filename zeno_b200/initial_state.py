"""Joint-space initial states for batched worlds (host side, numpy).

The reference's C ABI takes initial states as body poses and velocities
(``zeno_world_reset_to_state``, reference src/main.zig:357-394); reinforcement-learning
set-ups usually specify them as noise on joint coordinates (BASELINE-style "qpos / qvel
U(-a, a)").  ``joint_noise_state`` turns the second into the first by forward kinematics
over the model's own tables, so that it works for any loaded model:

* joints are visited in table order (a parent's joint comes before its children's);
* a hinge (type 1) rotates the child's subtree about the joint anchor
  (parent position + R(parent) anchor_parent) and the world axis R(parent) axis by an
  angle from U(-qpos, qpos); a slider (type 2) translates the subtree along its world axis
  by U(-qpos, qpos); a free joint (type 4) translates the subtree by U(-qpos, qpos) per
  axis and rotates it about the child's origin by a rotation vector with components
  U(-qpos, qpos); fixed and ball joints are left as they are;
* joint rates U(-qvel, qvel) give the subtree the matching rigid-body velocity.

Arithmetic is float64; the result is float32 in the ABI's float4 layout.
"""
from __future__ import annotations

import numpy as np

_BODY_FLOATS = 20   # BodyDataGPU: position, quaternion, inv_mass_inertia, params, com_offset
_JOINT_FLOATS = 20  # JointDataGPU: anchor_parent, anchor_child, axis, params, params2


def _axis_angle(axis, ang):
    h = 0.5 * ang
    return np.concatenate([axis * np.sin(h)[..., None], np.cos(h)[..., None]], -1)


def _qmul(a, b):
    ax, ay, az, aw = np.moveaxis(a, -1, 0)
    bx, by, bz, bw = np.moveaxis(b, -1, 0)
    return np.stack([aw * bx + ax * bw + ay * bz - az * by, aw * by - ax * bz + ay * bw + az * bx,
                     aw * bz + ax * by - ay * bx + az * bw, aw * bw - ax * bx - ay * by - az * bz], -1)


def _rot(q, v):
    qv, w = q[..., :3], q[..., 3:4]
    uv = np.cross(qv, v)
    return v + 2.0 * (w * uv + np.cross(qv, uv))


def joint_noise_state(bodies: bytes, joints: bytes, positions: np.ndarray, quaternions: np.ndarray,
                      num_envs: int, rng: np.random.Generator, qpos: float, qvel: float = 0.0) -> dict:
    """Body poses and velocities for ``num_envs`` environments: the single-environment pose
    (``positions`` / ``quaternions``, shape (B, 4), e.g. environment 0 of a fresh world)
    with joint-coordinate noise, from the model tables ``bodies`` and ``joints`` (the
    reference-layout records of ``ZenoWorld.model_table``).  Returns the four arrays
    ``zeno_world_reset_to_state`` takes, each (num_envs, B, 4) float32."""
    E = int(num_envs)
    bt = np.frombuffer(bodies, np.float32).reshape(-1, _BODY_FLOATS)
    B = bt.shape[0]
    jt = np.frombuffer(joints, np.float32).reshape(-1, _JOINT_FLOATS) if joints else np.zeros((0, _JOINT_FLOATS))
    pos = np.repeat(np.asarray(positions, np.float64).reshape(1, B, 4)[..., :3], E, axis=0)
    quat = np.repeat(np.asarray(quaternions, np.float64).reshape(1, B, 4), E, axis=0)
    vel = np.zeros((E, B, 3))
    ang = np.zeros((E, B, 3))
    parent = bt[:, 12].astype(np.int64)  # BodyDataGPU.params.x
    children = {b: [] for b in range(B)}
    for b in range(1, B):
        if 0 <= parent[b] < B and parent[b] != b:
            children[int(parent[b])].append(b)

    def subtree(b):
        out, todo = [], [b]
        while todo:
            x = todo.pop()
            out.append(x)
            todo.extend(children[x])
        return np.array(sorted(out))

    for j in jt:
        jtype, pa, ch = int(j[12]), int(j[13]), int(j[14])
        if jtype not in (1, 2, 4) or not 0 <= ch < B:
            continue
        sub = subtree(ch)
        if jtype == 4:
            d = rng.uniform(-qpos, qpos, size=(E, 3))
            rv = rng.uniform(-qpos, qpos, size=(E, 3))
            a = np.linalg.norm(rv, axis=1)
            r = _axis_angle(rv / np.maximum(a, 1e-30)[:, None], a)
            c0 = pos[:, ch:ch + 1].copy()
            pos[:, sub] = c0 + _rot(r[:, None], pos[:, sub] - c0) + d[:, None]
            quat[:, sub] = _qmul(r[:, None], quat[:, sub])
            continue
        axis_w = _rot(quat[:, pa], np.broadcast_to(j[8:11].astype(np.float64), (E, 3)))
        anchor = pos[:, pa] + _rot(quat[:, pa], np.broadcast_to(j[0:3].astype(np.float64), (E, 3)))
        x = rng.uniform(-qpos, qpos, size=E)
        xd = rng.uniform(-qvel, qvel, size=E) if qvel > 0 else np.zeros(E)
        if jtype == 1:
            n = axis_w / np.maximum(np.linalg.norm(axis_w, axis=1, keepdims=True), 1e-30)
            r = _axis_angle(n, x)
            pos[:, sub] = anchor[:, None] + _rot(r[:, None], pos[:, sub] - anchor[:, None])
            quat[:, sub] = _qmul(r[:, None], quat[:, sub])
            om = n * xd[:, None]
            ang[:, sub] += om[:, None]
            vel[:, sub] += np.cross(om[:, None], pos[:, sub] - anchor[:, None])
        else:
            pos[:, sub] += (axis_w * x[:, None])[:, None]
            vel[:, sub] += (axis_w * xd[:, None])[:, None]
    quat /= np.linalg.norm(quat, axis=-1, keepdims=True)

    def pad(a):
        return np.concatenate([a, np.zeros(a.shape[:-1] + (1,))], -1).astype(np.float32)

    return {"positions": pad(pos), "quaternions": quat.astype(np.float32), "velocities": pad(vel),
            "angular_velocities": pad(ang)}
