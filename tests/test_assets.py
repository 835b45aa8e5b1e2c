"""Every model the reference ships, and every sensor type its read_sensors kernel handles.

The reference's suite loads and steps each of its models (tests/test_python_integration.py:
661-701).  Here each one runs 10 steps (4 envs, seeded actions, one substep, the model's own
timestep) through the oracle, which must reproduce the committed golden rollout
(tests/golden/assets, made by tests/golden/make_asset_fixtures.py), and on the GPU, which
must match the oracle bit for bit, on both kernels.  Ant, Humanoid and the test pendulum are
covered by test_parity_gpu.py / test_golden.py.

Sensors: read_sensors (all_shaders.metal:1799-1893) handles joint position and velocity,
accelerometer (gravity in the body frame, R^-1 g), gyro, and frame position, quaternion,
linear and angular velocity.  The scene below declares all of them, under the reference
semantics (frame sensors observe body 0, so the accelerometer reads g and the gyro 0) and
under corrected semantics (sensors resolved by site to the moving body).
"""
from pathlib import Path

import numpy as np
import pytest

from parity import FIELDS, diff_report, product_state

ASSET_DIR = Path(__file__).resolve().parent / "golden" / "assets"
ASSETS = sorted(p.stem for p in ASSET_DIR.glob("*.xml"))

SENSOR_SCENE = """<mujoco model="sensors">
  <option timestep="0.01" gravity="0 0 -9.81"/>
  <worldbody>
    <geom type="plane" size="5 5 0.1"/>
    <body name="box" pos="0 0 0.4" euler="0.3 0.2 0.1">
      <joint name="free" type="free"/>
      <geom type="sphere" size="0.1" mass="1"/>
      <site name="imu" pos="0 0 0"/>
      <body name="arm" pos="0 0 0.1">
        <joint name="hinge" type="hinge" axis="0 1 0"/>
        <geom type="capsule" fromto="0 0 0 0.3 0 0" size="0.03" mass="0.2"/>
      </body>
    </body>
  </worldbody>
  <actuator>
    <motor joint="hinge" ctrlrange="-1 1" gear="5"/>
  </actuator>
  <sensor>
    <jointpos joint="hinge"/>
    <jointvel joint="hinge"/>
    <accelerometer site="imu"/>
    <gyro site="imu"/>
    <framepos objtype="site" objname="imu"/>
    <framequat objtype="site" objname="imu"/>
    <framelinvel objtype="site" objname="imu"/>
    <frameangvel objtype="site" objname="imu"/>
  </sensor>
</mujoco>
"""


def _load(name):
    xml = (ASSET_DIR / f"{name}.xml").read_text()
    d = np.load(ASSET_DIR / f"{name}_E4_N10.npz")
    return xml, d["actions"], {k: d[k] for k in FIELDS}


def test_all_shipped_models_present():
    assert ASSETS == ["cartpole", "cheetah", "hopper", "pusher", "reacher", "swimmer", "walker"]


@pytest.mark.parametrize("name", ASSETS)
def test_oracle_reproduces_asset_golden(name):
    from oracle.zeno_oracle import OracleWorld
    xml, acts, gold = _load(name)
    o = OracleWorld(xml, num_envs=4, substeps=1)
    for s in range(acts.shape[0]):
        o.step(acts[s])
    assert not diff_report(o.state(), gold)


def test_sensor_types_in_oracle():
    """The sensor scene declares every read_sensors type (0, 1, 2, 3, 7, 8, 9, 10)."""
    from oracle.zeno_oracle import OracleWorld
    o = OracleWorld(SENSOR_SCENE, num_envs=2, substeps=2)
    types = sorted(int(t) for t in o.raw("sensors", np.uint32).reshape(-1, 8)[:, 0])
    assert types == [0, 1, 2, 3, 7, 8, 9, 10]
    o.step(np.zeros((2, 1), np.float32))
    obs = o.state()["observations"]
    # reference semantics: frame sensors observe body 0 (identity pose, at rest)
    assert np.allclose(obs[:, 2:5], [0.0, 0.0, -9.81])  # accelerometer: R^-1 g with R = I
    assert np.all(obs[:, 5:8] == 0.0)                      # gyro of the static world body


@pytest.mark.gpu
@pytest.mark.parametrize("lanes", [1, 8])
@pytest.mark.parametrize("name", ASSETS)
def test_gpu_matches_oracle_and_golden_all_assets(name, lanes):
    from oracle.zeno_oracle import OracleWorld
    from zeno_b200 import ZenoWorld
    xml, acts, gold = _load(name)
    w = ZenoWorld(mjcf_string=xml, num_envs=4, substeps=1)
    if lanes != w.get_launch()[0]:
        w.set_launch(lanes, 4)
    o = OracleWorld(xml, num_envs=4, substeps=1)
    for s in range(acts.shape[0]):
        w.step(acts[s])
        o.step(acts[s])
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"{name} (lanes {lanes}) step {s + 1}: {bad}"
    assert not diff_report(product_state(w), gold)


@pytest.mark.gpu
@pytest.mark.parametrize("semantics", ["reference", "corrected"])
def test_gpu_sensor_types_bit_exact(semantics):
    from oracle.zeno_oracle import OracleWorld
    from zeno_b200 import ZenoWorld
    E = 8
    kw = dict(num_envs=E, substeps=2, max_contacts_per_env=16, semantics=semantics)
    w = ZenoWorld(mjcf_string=SENSOR_SCENE, **kw)
    o = OracleWorld(SENSOR_SCENE, **kw)
    rng = np.random.default_rng(5)
    for s in range(10):
        a = rng.uniform(-1, 1, size=(E, 1)).astype(np.float32)
        w.step(a)
        o.step(a)
        if s in (0, 9):
            bad = diff_report(product_state(w), o.state())
            assert not bad, f"{semantics} step {s + 1}: {bad}"
    obs = w.get_observations()
    if semantics == "corrected":  # the IMU rides the free body: tilted gravity, non-zero rates
        assert np.abs(obs[:, 2:5] - np.array([0.0, 0.0, -9.81])).max() > 1e-3
        assert np.abs(obs[:, 5:8]).max() > 0.0
