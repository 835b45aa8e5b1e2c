"""Golden rollouts (tests/golden/*.npz, made by tests/golden/make_golden.py): the oracle must
keep reproducing them (CPU), and the GPU step must match them bit for bit (GPU)."""
from pathlib import Path

import numpy as np
import pytest

from parity import CONFIGS, FIELDS, diff_report, product_state

GOLD = Path(__file__).resolve().parent / "golden"
CASES = [(n, False) for n in CONFIGS] + [("ant", True)]


def load(name, task):
    f = GOLD / (f"ant_task_E4_N10.npz" if task else f"{name}_E4_N10.npz")
    d = np.load(f)
    return d["actions"], {k: d[k] for k in FIELDS}


def run(world, acts, task):
    if task:
        world.set_task(body=1, z_min=0.2, z_max=1.0, auto_reset=True, noise=0.1, seed=5)
    for s in range(acts.shape[0]):
        world.step(acts[s])


@pytest.mark.parametrize("name,task", CASES)
def test_oracle_reproduces_golden(name, task):
    from oracle.zeno_oracle import OracleWorld
    c = CONFIGS[name]
    acts, gold = load(name, task)
    o = OracleWorld(c["xml"](), num_envs=4, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
                    max_contacts_per_env=c["max_contacts"], substeps=c["substeps"])
    run(o, acts, task)
    assert not diff_report(o.state(), gold)


@pytest.mark.gpu
@pytest.mark.parametrize("name,task", CASES)
def test_gpu_matches_golden(name, task):
    from zeno_b200 import ZenoWorld
    c = CONFIGS[name]
    acts, gold = load(name, task)
    w = ZenoWorld(mjcf_string=c["xml"](), num_envs=4, timestep=c.get("timestep", 0.0), contact_iterations=c["iters"],
                  max_contacts_per_env=c["max_contacts"], substeps=c["substeps"])
    run(w, acts, task)
    assert not diff_report(product_state(w), gold)
