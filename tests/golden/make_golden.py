"""Regenerate the golden rollouts in tests/golden/*.npz with the CPU oracle.

The reference pins no trajectories (its step runs under Metal fast-math), so these
fixtures are produced by the oracle, which is itself pinned to the reference's known
answers (tests/test_oracle_known_answers.py).  They freeze the oracle's results so a
change to either implementation is caught even where the oracle is not rebuilt, and give
the GPU tests a fixed target.

    python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE.parent))

from oracle.zeno_oracle import OracleWorld  # noqa: E402
from parity import CONFIGS, actions  # noqa: E402

E, N = 4, 10


def rollout(name, task=False):
    c = CONFIGS[name]
    xml = c["xml"]()
    o = OracleWorld(xml, num_envs=E, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
                    max_contacts_per_env=c["max_contacts"], substeps=c["substeps"])
    if task:
        o.set_task(body=1, z_min=0.2, z_max=1.0, auto_reset=True, noise=0.1, seed=5)
    a = actions(np.random.default_rng(2024), N, E, o.num_actuators, c["act"])
    for s in range(N):
        o.step(a[s])
    return a, o.state()


def main():
    for name in CONFIGS:
        a, st = rollout(name)
        np.savez_compressed(HERE / f"{name}_E{E}_N{N}.npz", actions=a, **st)
    a, st = rollout("ant", task=True)
    np.savez_compressed(HERE / f"ant_task_E{E}_N{N}.npz", actions=a, **st)
    print("written")


if __name__ == "__main__":
    main()
