"""Pin the CPU oracle to every known answer the reference's tests hold for this path.

The reference ships no trajectory goldens (its GPU step runs under Metal fast-math);
these are the values its unit tests assert, re-checked here against the oracle:
  tests/test_mjcf.zig:371-496         MJCF mass / inertia / option parsing
  tests/test_physics_integration.zig  joint decomposition counts (16-194), effective mass
                                      (405-475), actuator torque and clamps (517-629)
  tests/test_collision.zig            sphere-sphere / sphere-plane penetration (55-69, 173-187)
  tests/test_xpbd.zig:370-376         record sizes
plus the Ant model derived by hand from the reference loader (B=10, J=9, K=24,
obs=29, 12 colours of sizes 4,4,4,2,2,2,1,1,1,1,1,1)."""
import ctypes
import struct

import numpy as np
import pytest

from oracle.zeno_oracle import OracleWorld, lib
from zeno_b200 import scenes


def bodies(o):
    """BodyDataGPU records: (position, quaternion, inv_mass_inertia, params, com_offset)."""
    raw = o.raw("bodies")
    return raw.reshape(-1, 5, 4)


def mjcf(body_xml, option='<option timestep="0.01" gravity="0 0 -10"/>', extra=""):
    return f'<mujoco model="t">{option}<worldbody>{body_xml}</worldbody>{extra}</mujoco>'


def test_option_parsing():
    # test_mjcf.zig: timestep 0.01 / gravity -10
    o = OracleWorld(mjcf('<geom type="plane" size="5 5 0.1"/><body name="ball" pos="0 0 1"><joint type="free"/>'
                         '<geom type="sphere" size="0.1" mass="1"/></body>'))
    assert o.num_bodies == 2  # world + ball
    o.step(np.zeros((1, 0), np.float32))
    acc = o.state()["accelerations"][0, 1]
    # one substep of free fall: dv = g*dt*0.999 over one timestep -> a = -10 * 0.999
    assert acc[2] == pytest.approx(-10 * 0.999, rel=1e-4)  # v is re-derived from positions (XPBD)


def test_explicit_inertial():
    o = OracleWorld(mjcf('<body name="heavy" pos="0 0 1"><inertial mass="5.0" pos="0 0 0" diaginertia="0.1 0.2 0.3"/>'
                         '<joint type="free"/><geom type="sphere" size="0.1"/></body>'))
    b = bodies(o)[1]
    assert 1 / b[2][0] == pytest.approx(5.0, abs=1e-3)
    assert 1 / b[2][1] == pytest.approx(0.1, abs=1e-3)
    assert 1 / b[2][2] == pytest.approx(0.2, abs=1e-3)
    assert 1 / b[2][3] == pytest.approx(0.3, abs=1e-3)


def test_mass_from_geom_mass():
    o = OracleWorld(mjcf('<body name="ball" pos="0 0 1"><joint type="free"/><geom type="sphere" size="0.1" mass="2.5"/></body>'))
    b = bodies(o)[1]
    assert 1 / b[2][0] == pytest.approx(2.5, abs=1e-3)
    assert 1 / b[2][1] == pytest.approx(0.01, abs=1e-3)  # 0.4 m r^2


def test_mass_from_density():
    o = OracleWorld(mjcf('<body name="ball" pos="0 0 1"><joint type="free"/><geom type="sphere" size="0.1" density="500"/></body>'))
    b = bodies(o)[1]
    assert 1 / b[2][0] == pytest.approx(2.094, abs=0.05)
    assert b[2][1] > 0


def test_composite_inertia():
    o = OracleWorld(mjcf('<body name="c" pos="0 0 1"><joint type="free"/>'
                         '<geom type="sphere" size="0.1" mass="1.0" pos="0 0 0"/>'
                         '<geom type="sphere" size="0.1" mass="1.0" pos="0.5 0 0"/></body>'))
    b = bodies(o)[1]
    assert 1 / b[2][0] == pytest.approx(2.0, abs=1e-3)
    Ixx, Iyy, Izz = 1 / b[2][1], 1 / b[2][2], 1 / b[2][3]
    assert Iyy > Ixx and Izz > Ixx
    assert b[4][0] == pytest.approx(0.25)  # centre of mass offset


def test_box_inertia():
    o = OracleWorld(mjcf('<body name="block" pos="0 0 1"><joint type="free"/><geom type="box" size="0.5 0.3 0.1" mass="6.0"/></body>'))
    b = bodies(o)[1]
    assert 1 / b[2][0] == pytest.approx(6.0, abs=1e-3)
    assert 1 / b[2][1] == pytest.approx(0.2, abs=0.01)
    assert 1 / b[2][2] == pytest.approx(0.52, abs=0.01)
    assert 1 / b[2][3] == pytest.approx(0.68, abs=0.01)


@pytest.mark.parametrize("joint,expected", [
    ('<joint type="hinge" axis="0 0 1"/>', [2, 3]),                                   # point + hinge
    ('<joint type="hinge" axis="0 0 1" range="-1.57 1.57"/>', [2, 3, 4]),             # + angular limit
    ("", [7]),                                                                        # fixed -> weld
    ('<joint type="ball"/>', [2]),                                                    # point only
    ('<joint type="ball" range="0 0.5"/>', [2, 4]),                                   # + cone limit
    ('<joint type="slide" axis="1 0 0"/>', [10]),                                     # slider
    ('<joint type="slide" axis="1 0 0" range="-1 1"/>', [10, 5]),                     # + linear limit
    ('<joint type="free"/>', []),                                                     # nothing
])
def test_joint_decomposition(joint, expected):
    o = OracleWorld(mjcf(f'<body name="b" pos="0 0 1">{joint}<geom type="sphere" size="0.1"/></body>'))
    t = o.raw("constraint_template", np.uint32).reshape(-1, 24)
    types = sorted(int(x) & 0xFF for x in t[:, 3]) if t.size else []
    assert types == sorted(expected)


def test_cone_limit_is_symmetric():
    o = OracleWorld(mjcf('<body name="b" pos="0 0 1"><joint type="ball" range="0 0.5"/><geom type="sphere" size="0.1"/></body>'))
    t = o.raw("constraint_template").reshape(-1, 24)
    lim = [r for r in t if (r.view(np.uint32)[3] & 0xFF) == 4][0]
    assert lim[16] == pytest.approx(-0.5) and lim[17] == pytest.approx(0.5)


def _w(ima, imb, Ia, Ib, ra, rb, n):
    f3 = lambda v: (ctypes.c_float * 3)(*v)
    L = lib()
    L.zo_effective_mass.restype = ctypes.c_float
    return L.zo_effective_mass(ctypes.c_float(ima), ctypes.c_float(imb), f3(Ia), f3(Ib), f3(ra), f3(rb), f3(n))


def test_effective_mass_known_answers():
    assert _w(1, 1, (1, 1, 1), (1, 1, 1), (0, 0, 0), (0, 0, 0), (1, 0, 0)) == pytest.approx(2.0)
    assert _w(1, 1, (1, 1, 1), (1, 1, 1), (0, 1, 0), (0, -1, 0), (1, 0, 0)) == pytest.approx(4.0)
    assert _w(0, 1, (0, 0, 0), (1, 1, 1), (0, 0, 0), (0, 0, 0), (0, 0, 1)) == pytest.approx(1.0)


def _actuated(motor_attrs):
    return mjcf('<body name="arm" pos="0 0 1"><joint name="j" type="hinge" axis="0 0 1"/><geom type="sphere" size="0.1"/></body>',
                extra=f'<actuator><motor joint="j" {motor_attrs}/></actuator>')


@pytest.mark.parametrize("attrs,ctrl,torque", [
    ('gear="10" ctrlrange="-1 1" forcerange="-100 100"', 0.5, 5.0),     # torque = ctrl * gear
    ('gear="10" ctrlrange="-1 1" forcerange="-100 100"', 5.0, 10.0),    # ctrl clamped to 1
    ('gear="1000" ctrlrange="-1 1" forcerange="-50 50"', 1.0, 50.0),    # force clamp
    ('gear="100" ctrlrange="-1 1"', 1.0, 100.0),                        # unbounded force range
    ('gear="100" ctrlrange="-1 1"', -1.0, -100.0),
    ('gear="100" ctrlrange="-1 1"', 0.5, 50.0),
])
def test_actuator_torques(attrs, ctrl, torque):
    o = OracleWorld(_actuated(attrs))
    o.step(np.array([[ctrl]], np.float32))
    assert o.state()["joint_torques"][0, 0] == pytest.approx(torque, abs=0.01)


def _contact_world(bodies_xml):
    return OracleWorld(mjcf(bodies_xml, option='<option timestep="0.01" gravity="0 0 0"/>'))


def test_sphere_sphere_penetration_and_normal():
    o = _contact_world('<body name="a" pos="0 0 0"><joint type="free"/><geom type="sphere" size="0.5"/></body>'
                       '<body name="b" pos="0.8 0 0"><joint type="free"/><geom type="sphere" size="0.5"/></body>')
    o.step(np.zeros((1, 0), np.float32))
    c = o.state()["contacts"][0, 0]
    assert c["position_pen"][3] == pytest.approx(0.2, abs=0.01)
    assert c["normal_friction"][0] == pytest.approx(1.0, abs=0.01)


def test_sphere_plane_penetration():
    o = _contact_world('<geom type="plane" size="5 5 0.1"/>'
                       '<body name="s" pos="0 0 0.3"><joint type="free"/><geom type="sphere" size="0.5"/></body>')
    o.step(np.zeros((1, 0), np.float32))
    c = o.state()["contacts"][0, 0]
    assert c["position_pen"][3] == pytest.approx(0.2, abs=0.01)


def test_record_sizes():
    # XPBDConstraint 96 B, ContactGPU 64 B, BodyDataGPU 80 B, JointDataGPU 80 B, GeomGPU 64 B
    o = OracleWorld(scenes.ant())
    assert len(o.model_table("constraint_template")) == 96 * o.num_constraints
    assert o.state()["contacts"].dtype.itemsize == 64
    assert len(o.model_table("bodies")) == 80 * o.num_bodies
    assert len(o.model_table("joints")) == 80 * o.num_joints
    assert len(o.model_table("geoms")) == 64 * o.num_geoms


def test_ant_model_as_derived_from_the_reference_loader():
    o = OracleWorld(scenes.ant())
    assert (o.num_bodies, o.num_joints, o.num_actuators, o.num_geoms) == (10, 9, 8, 10)
    assert (o.num_constraints, o.obs_dim, o.num_colors) == (24, 29, 12)
    ranges = o.raw("color_ranges", np.uint32).reshape(-1, 2)
    assert ranges[:, 1].tolist() == [4, 4, 4, 2, 2, 2, 1, 1, 1, 1, 1, 1]
    # frame sensors observe body 0 (world): pos 0, quat identity, velocities 0
    o.step(np.zeros((1, 8), np.float32))
    obs = o.state()["observations"][0]
    assert obs[:13].tolist() == [0, 0, 0, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0]


def test_humanoid_model_sizes():
    o = OracleWorld(scenes.humanoid())
    assert (o.num_bodies, o.num_joints, o.num_actuators, o.num_geoms) == (15, 14, 13, 15)
    assert (o.num_constraints, o.obs_dim) == (39, 39)


def test_contact_counter_grows_and_list_freezes():
    """Reference: contact_counts is never reset by the step (only by reset), slots past
    max_contacts are never written (all_shaders.metal:525-531)."""
    o = OracleWorld(scenes.ant(), num_envs=2, substeps=1)
    a = np.zeros((2, 8), np.float32)
    o.step(a)
    # 9 plane pairs + 4 torso-hip pairs pass the broad phase in the initial pose
    assert (o.state()["contact_counts"] == 13).all()
    prev = 13
    for _ in range(12):
        o.step(a)
        c = o.state()["contact_counts"]
        assert (c > prev).all()
        prev = c.min()
    assert prev > 64  # the counter keeps growing past max_contacts; the 64 slots froze
    o.reset()
    assert (o.state()["contact_counts"] == 0).all()
