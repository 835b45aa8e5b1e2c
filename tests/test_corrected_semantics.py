"""Corrected semantics (ZENO_SEMANTICS_CORRECTED; no counterpart in the reference): the
MJCF compiler rules the reference loader skips, and the step conventions that make
resting contact hold.  The product loader and the oracle's are separate implementations
whose model tables must be byte-identical; known answers below are derived by hand from
the MJCF rules; the resting-contact checks run on the oracle (CPU)."""
import numpy as np
import pytest

from oracle.zeno_oracle import OracleWorld
from zeno_b200 import _ffi, scenes

from test_model_tables import EXTRA, ORACLE_NAMES

S = float(np.sqrt(0.5))
DEG = np.float32(0.017453292519943295)

CORRECTED_EXTRA = {
    "rotated_parent": '<mujoco><worldbody><body name="p" pos="0 0 1" euler="0 0 90"><joint type="free"/>'
                      '<geom type="sphere" size="0.1"/><body name="c" pos="1 0 0"><joint name="h" type="hinge" '
                      'pos="0.5 0 0" axis="2 0 0" range="-30 45"/><geom type="box" size="0.5 0.1 0.1"/>'
                      '</body></body></worldbody></mujoco>',
    "radian_xyz_upper": '<mujoco><compiler angle="radian" eulerseq="XYZ"/><worldbody><body name="r" pos="0 0 1" '
                        'euler="0.3 0.2 0.1"><joint type="hinge" range="-1 1"/><geom type="capsule" '
                        'fromto="0 0 0 0.4 0 0" size="0.05"/></body></worldbody></mujoco>',
    "sensors_by_name": '<mujoco><worldbody><body name="torso" pos="0 0 1"><joint type="free"/><geom type="sphere" '
                       'size="0.1"/><body name="arm" pos="0.2 0 0"><joint name="j" type="hinge"/><site name="tip" '
                       'pos="0.1 0 0"/><geom type="capsule" fromto="0 0 0 0.2 0 0" size="0.02"/></body></body>'
                       '</worldbody><sensor><framepos objtype="body" objname="arm"/><framequat objname="torso"/>'
                       '<accelerometer site="tip"/><jointpos joint="j"/></sensor></mujoco>',
    "cylinder_fromto": '<mujoco><worldbody><body name="b" pos="0 0 1"><joint type="free"/><geom type="cylinder" '
                       'fromto="0 0 0 0 0.6 0" size="0.05"/></body></worldbody></mujoco>',
}


def tables(xml, sem):
    t = _ffi.model_tables(xml, sem)
    return {
        "bodies": np.frombuffer(t["bodies"], np.float32).reshape(-1, 20),
        "joints": np.frombuffer(t["joints"], np.float32).reshape(-1, 20),
        "geoms": np.frombuffer(t["geoms"], np.float32).reshape(-1, 16),
        "sensors": np.frombuffer(t["sensors"], np.uint32).reshape(-1, 8),
    }


ALL = {**{k: v for k, v in scenes.BY_NAME.items()}, **{k: (lambda x=v: x) for k, v in EXTRA.items()},
       **{k: (lambda x=v: x) for k, v in CORRECTED_EXTRA.items()}}


@pytest.mark.parametrize("name", list(ALL))
def test_corrected_tables_match_oracle(name):
    xml = ALL[name]()
    ours = _ffi.model_tables(xml, "corrected")
    o = OracleWorld(xml, semantics="corrected")
    for k, on in ORACLE_NAMES.items():
        assert ours[k] == o.model_table(on), f"{name}: table {k} differs"


def test_parent_rotation_composes():
    """Parent at (0,0,1) turned 90 degrees about z (euler in degrees): the child's pos
    (1,0,0) lands at (0,1,1) and it inherits the parent's orientation; the reference adds
    the offset unrotated, at (1,0,1), and takes euler="0 0 90" as 90 radians."""
    c = tables(CORRECTED_EXTRA["rotated_parent"], "corrected")
    np.testing.assert_allclose(c["bodies"][2, 0:3], (0, 1, 1), atol=1e-6)
    np.testing.assert_allclose(c["bodies"][1, 4:8], (0, 0, S, S), atol=1e-6)
    np.testing.assert_allclose(c["bodies"][2, 4:8], (0, 0, S, S), atol=1e-6)
    r = tables(CORRECTED_EXTRA["rotated_parent"], "reference")
    np.testing.assert_allclose(r["bodies"][2, 0:3], (1, 0, 1), atol=1e-6)


def test_joint_frame_and_degrees():
    """Joint pos/axis are child-frame: anchor_parent = child pos + R_local jpos, axis
    normalised (2,0,0) -> (1,0,0) (the child has no rotation of its own here); hinge range
    in degrees -> radians."""
    c = tables(CORRECTED_EXTRA["rotated_parent"], "corrected")
    j = c["joints"][1]
    np.testing.assert_allclose(j[0:3], (1.5, 0, 0), atol=1e-6)  # anchor_parent
    np.testing.assert_allclose(j[4:7], (0.5, 0, 0), atol=1e-6)  # anchor_child
    np.testing.assert_allclose(j[8:11], (1, 0, 0), atol=1e-6)  # axis
    assert j[15] == np.float32(-30) * DEG
    r = tables(CORRECTED_EXTRA["rotated_parent"], "reference")
    assert r["joints"][1, 15] == -30 and r["joints"][1, 8] == 2


def test_radian_and_fixed_axes_and_fromto():
    """angle="radian" keeps ranges and angles as written; eulerseq "XYZ" (fixed axes)
    composes z(0.1) y(0.2) x(0.3); a fromto capsule along +x turns local z onto x and sits
    at the segment midpoint."""
    c = tables(CORRECTED_EXTRA["radian_xyz_upper"], "corrected")
    assert c["joints"][0, 15] == np.float32(-1)

    def qaxis(ax, a):
        q = np.zeros(4)
        q[ax] = np.sin(a / 2)
        q[3] = np.cos(a / 2)
        return q

    def qmul(a, b):
        ax, ay, az, aw = a
        bx, by, bz, bw = b
        return np.array([aw * bx + ax * bw + ay * bz - az * by, aw * by - ax * bz + ay * bw + az * bx,
                         aw * bz + ax * by - ay * bx + az * bw, aw * bw - ax * bx - ay * by - az * bz])

    want = qmul(qaxis(2, 0.1), qmul(qaxis(1, 0.2), qaxis(0, 0.3)))
    np.testing.assert_allclose(c["bodies"][1, 4:8], want, atol=1e-6)
    g = c["geoms"][0]
    np.testing.assert_allclose(g[4:7], (0.2, 0, 0), atol=1e-6)       # centre
    np.testing.assert_allclose(g[8:12], (0, S, 0, S), atol=1e-6)     # +z onto +x


def test_cylinder_fromto_and_rotated_inertia():
    """A cylinder along y (fromto) has half length 0.3 and its axial (smaller) moment on
    the body's y axis, not z."""
    c = tables(CORRECTED_EXTRA["cylinder_fromto"], "corrected")
    g = c["geoms"][0]
    assert abs(g[12] - 0.3) < 1e-6  # size[1]
    inv_i = c["bodies"][1, 8:12]    # 1/m, 1/Ixx, 1/Iyy, 1/Izz
    assert inv_i[2] > 10 * inv_i[1] and abs(inv_i[1] - inv_i[3]) < 1e-3 * inv_i[1]


def test_sensors_resolve_their_body():
    c = tables(CORRECTED_EXTRA["sensors_by_name"], "corrected")
    obj = c["sensors"][:, 1]
    assert list(obj[:3]) == [2, 1, 2]  # framepos arm, framequat torso, accelerometer site on arm
    r = tables(CORRECTED_EXTRA["sensors_by_name"], "reference")
    assert list(r["sensors"][:3, 1]) == [0, 0, 0]


def test_automatic_sensors_observe_the_root_body():
    """Without <sensor>, the reference's automatic frame sensors observe body 0 (world);
    corrected, the world's first child (the Ant torso)."""
    xml = scenes.ant()
    assert set(tables(xml, "reference")["sensors"][:4, 1]) == {0}
    assert set(tables(xml, "corrected")["sensors"][:4, 1]) == {1}


RESTING = {
    "sphere": '<body pos="0 0 0.1"><joint type="free"/><geom type="sphere" size="0.1"/></body>',
    "sphere_stack": '<body pos="0 0 0.1"><joint type="free"/><geom type="sphere" size="0.1"/></body>'
                    '<body pos="0 0 0.3"><joint type="free"/><geom type="sphere" size="0.1"/></body>',
    "capsule_lying": '<body pos="0 0 0.05" euler="0 90 0"><joint type="free"/><geom type="capsule" '
                     'size="0.05 0.2"/></body>',
    "box_stack": '<body pos="0 0 0.1"><joint type="free"/><geom type="box" size="0.1 0.1 0.1"/></body>'
                 '<body pos="0 0 0.3"><joint type="free"/><geom type="box" size="0.1 0.1 0.1"/></body>',
    "capsule_on_box": '<body pos="0 0 0.1"><joint type="free"/><geom type="box" size="0.2 0.2 0.1"/></body>'
                      '<body pos="0 0 0.25" euler="90 0 0"><joint type="free"/><geom type="capsule" '
                      'size="0.05 0.15"/></body>',
}


def resting_xml(bodies):
    return ('<mujoco><option timestep="0.005"/><worldbody><geom type="plane" size="5 5 .1"/>' + bodies +
            '</worldbody></mujoco>')


@pytest.mark.parametrize("name", list(RESTING))
def test_resting_contact_holds(name):
    """Bodies placed in touching contact stay at rest under corrected semantics (one slot
    per touching pair, normals from B to A); under the reference's semantics the frozen,
    duplicated slot list launches them."""
    xml = resting_xml(RESTING[name])
    z0 = None
    for sem in ("corrected", "reference"):
        o = OracleWorld(xml, num_envs=1, substeps=8, max_contacts_per_env=32, semantics=sem)
        assert o.set_narrow_phase(2) == 0
        for _ in range(200):
            o.step(np.zeros((1, 0), np.float32))
        st = o.state()
        z = st["positions"][0, 1:, 2]
        if sem == "corrected":
            z0 = z
            assert np.abs(st["velocities"][0, 1:, :3]).max() < 0.05
            assert np.all(z > 0) and np.all(z < 0.35)
        else:
            assert z.max() > 0.5, "the reference's frozen slot list should launch the bodies"
    assert z0 is not None


def test_corrected_refuses_the_gpu_narrow_phase():
    o = OracleWorld(scenes.ant(), semantics="corrected")
    assert o.set_narrow_phase(0) != 0
    assert o.set_narrow_phase(1) == 0 and o.set_narrow_phase(2) == 0
