"""Model fixtures for the all-assets parity test, made in a container that holds the
reference checkout (the GPU box does not).

The reference's suite loads and steps every model it ships (tests/test_python_integration.py:
661-701, assets/*.xml).  The Ant, Humanoid and test pendulum are already in
zeno_b200/scenes.py; this script writes the other shipped models (cartpole, cheetah,
hopper, pusher, reacher, swimmer, walker) as model data under tests/golden/assets/, with
XML comments and rgba attributes removed (they do not reach the step), and records a
10-step oracle rollout of each (4 envs, seeded actions) next to it as a golden fixture.

    python tests/golden/make_asset_fixtures.py <path of the reference checkout>
"""
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE.parent))

from oracle.zeno_oracle import OracleWorld  # noqa: E402

ASSETS = ("cartpole", "cheetah", "hopper", "pusher", "reacher", "swimmer", "walker")
E, N = 4, 10


def normalise(xml: str) -> str:
    xml = re.sub(r"<!--.*?-->", "", xml, flags=re.S)
    xml = re.sub(r'\s+rgba="[^"]*"', "", xml)
    return "\n".join(line.rstrip() for line in xml.splitlines() if line.strip()) + "\n"


def rollout(xml: str):
    o = OracleWorld(xml, num_envs=E, substeps=1)
    a = np.random.default_rng(7).uniform(-1, 1, size=(N, E, max(o.num_actuators, 1))).astype(np.float32)
    for s in range(N):
        o.step(a[s])
    return a, o.state()


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_asset_fixtures.py <path of the reference checkout>")
    ref = Path(sys.argv[1])
    out = HERE / "assets"
    out.mkdir(exist_ok=True)
    for name in ASSETS:
        xml = normalise((ref / "assets" / f"{name}.xml").read_text())
        (out / f"{name}.xml").write_text(xml)
        a, st = rollout(xml)
        np.savez_compressed(out / f"{name}_E{E}_N{N}.npz", actions=a, **st)
        print(name, len(xml), "bytes")


if __name__ == "__main__":
    main()
