"""The product's MJCF loader and model builder (zeno_b200/csrc/mjcf.cpp, model.cpp) are a
separate implementation from the oracle's; their model tables -- BodyDataGPU, JointDataGPU,
GeomGPU, ActuatorDataGPU, SensorGPU records, the colour-sorted XPBDConstraint template and
the colour ranges -- must be byte-identical (host only, no GPU needed)."""
import pytest

from oracle.zeno_oracle import OracleWorld
from zeno_b200 import _ffi, scenes

ORACLE_NAMES = {"bodies": "bodies", "joints": "joints", "geoms": "geoms", "actuators": "actuators",
                "sensors": "sensors", "constraints": "constraint_template", "color_ranges": "color_ranges"}

EXTRA = {
    # reference tests/test_mjcf.zig fixtures (restated)
    "inertial": '<mujoco><worldbody><body name="h" pos="0 0 1"><inertial mass="5.0" pos="0 0 0" '
                'diaginertia="0.1 0.2 0.3"/><joint type="free"/><geom type="sphere" size="0.1"/></body></worldbody></mujoco>',
    "nested": '<mujoco><worldbody><body name="b1" pos="0 0 1"><geom type="sphere" size="0.1"/><body name="b2" pos="0 0 1">'
              '<geom type="sphere" size="0.1"/><body name="b3" pos="0 0 1"><geom type="sphere" size="0.1"/>'
              '</body></body></body></worldbody></mujoco>',
    "euler": '<mujoco><worldbody><body name="r" pos="0 0 1" euler="90 0 0"><geom type="box" size="0.5 0.1 0.1"/>'
             '</body></worldbody></mujoco>',
    "quat": '<mujoco><worldbody><body name="r" pos="0 0 1" quat="0.707 0 0.707 0"><joint type="hinge" axis="1 0 0"/>'
            '<geom type="box" size="0.5 0.1 0.1"/></body></worldbody></mujoco>',
    "defaults_classes": '<mujoco><default><geom friction="0.5 0.1 0.1" density="300"/><joint damping="0.5"/>'
                        '<default class="leg"><geom type="capsule" size="0.04 0.2"/></default></default>'
                        '<worldbody><body name="b" pos="0 0 1" childclass="leg"><joint type="hinge" range="-1 1"/>'
                        '<geom/><geom class="main" type="sphere" size="0.1"/></body></worldbody></mujoco>',
    "slider_limits": '<mujoco><worldbody><body name="c" pos="0 0 1"><joint name="s" type="slide" axis="1 0 0" '
                     'range="-1 1"/><geom type="box" size="0.1 0.1 0.1"/></body></worldbody>'
                     '<actuator><motor joint="s" gear="5" forcerange="-3 3"/></actuator></mujoco>',
    "ball_cone": '<mujoco><worldbody><body name="b" pos="0 0 1"><joint type="ball" range="0 0.7"/>'
                 '<geom type="cylinder" size="0.05 0.2"/></body></worldbody></mujoco>',
    "autosensors": '<mujoco><worldbody><body name="b" pos="0 0 1"><joint name="a" type="hinge"/><joint name="b2" '
                   'type="hinge" axis="1 0 0"/><geom type="sphere" size="0.1" mass="0"/></body></worldbody></mujoco>',
    "comments_and_quirks": '<?xml version="1.0"?><mujoco model="q"><!-- a comment --><option timestep="0.005"/>'
                           '<worldbody><geom type="plane"/><body pos="0 0  1"><geom type="sphere" size="0.1  0.2" '
                           'friction="0.8"/></body></worldbody></mujoco>',
}


@pytest.mark.parametrize("name", list(scenes.BY_NAME) + list(EXTRA))
def test_model_tables_match_oracle(name):
    xml = scenes.BY_NAME[name]() if name in scenes.BY_NAME else EXTRA[name]
    ours = _ffi.model_tables(xml)
    o = OracleWorld(xml)
    for k, on in ORACLE_NAMES.items():
        assert ours[k] == o.model_table(on), f"{name}: table {k} differs"
