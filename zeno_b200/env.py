"""``ZenoEnv`` and ``make``: the reference's batched environment wrapper
(python/zeno/env.py:13-267 in Lulzx/zeno) over the sm_100a world."""
from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import numpy as np

from . import scenes
from ._ffi import ZenoWorld


class ZenoEnv:
    """Batched environment: reset(mask) -> obs; step(actions) -> (obs, rewards, dones, info)."""

    def __init__(self, mjcf_path: Optional[str] = None, mjcf_string: Optional[str] = None, num_envs: int = 1,
                 timestep: float = 0, contact_iterations: int = 4, max_contacts_per_env: int = 64,
                 seed: int = 42, substeps: int = 1):
        self._world = ZenoWorld(mjcf_path=mjcf_path, mjcf_string=mjcf_string, num_envs=num_envs,
                                timestep=timestep, contact_iterations=contact_iterations,
                                max_contacts_per_env=max_contacts_per_env, seed=seed, substeps=substeps)
        self._num_envs = num_envs
        self._step_count = 0
        self._max_episode_steps = 1000
        self._mjcf_path = mjcf_path
        self._obs_shape = (num_envs, self._world.obs_dim)
        self._action_shape = (num_envs, self._world.action_dim)

    num_envs = property(lambda self: self._num_envs)
    observation_dim = property(lambda self: self._world.obs_dim)
    action_dim = property(lambda self: self._world.action_dim)
    timestep = property(lambda self: self._world.timestep)
    observation_shape = property(lambda self: self._obs_shape)
    action_shape = property(lambda self: self._action_shape)
    world = property(lambda self: self._world)

    def reset(self, mask: Optional[np.ndarray] = None) -> np.ndarray:
        self._world.reset(mask)
        self._step_count = 0
        return self._world.get_observations().copy()

    def step(self, actions: np.ndarray, substeps: int = 0) -> Tuple[np.ndarray, np.ndarray, np.ndarray, Dict[str, Any]]:
        actions = np.asarray(actions, dtype=np.float32)
        if actions.shape != self._action_shape:
            actions = actions.reshape(self._action_shape)
        self._world.step(actions, substeps)
        self._step_count += 1
        obs = self._world.get_observations().copy()
        rewards = self._world.get_rewards()
        dones = self._world.get_dones()
        truncated = np.zeros(self._num_envs, dtype=bool)
        if self._step_count >= self._max_episode_steps:
            truncated[:] = True
        return obs, rewards, dones.astype(bool), {"step_count": self._step_count, "truncated": truncated}

    def get_body_positions(self) -> np.ndarray:
        return self._world.get_body_positions()

    def get_body_quaternions(self) -> np.ndarray:
        return self._world.get_body_quaternions()

    def close(self) -> None:
        pass

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()


def make(model: str, num_envs: int = 1, **kwargs) -> ZenoEnv:
    """Create an environment from an MJCF path, or from a built-in model name
    (ant, humanoid, pendulum, cartpole, pendulum_asset, collision_stress)."""
    path = Path(model)
    if path.exists():
        return ZenoEnv(mjcf_path=str(path), num_envs=num_envs, **kwargs)
    name = model[:-4] if model.endswith(".xml") else model
    if name in scenes.BY_NAME:
        return ZenoEnv(mjcf_string=scenes.BY_NAME[name](), num_envs=num_envs, **kwargs)
    for d in (Path.cwd() / "assets", Path.home() / ".zeno" / "assets"):
        p = d / f"{name}.xml"
        if p.exists():
            return ZenoEnv(mjcf_path=str(p), num_envs=num_envs, **kwargs)
    raise FileNotFoundError(f"Could not find model '{model}'")
