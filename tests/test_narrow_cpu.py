"""The extended narrow phase (the reference's CPU detectCollision, restated in
oracle/oracle_narrow.cpp) against the known answers of the reference's own tests
(tests/test_collision.zig:55-81, 173-199, 219-232; src/collision/gjk.zig:712-826 for GJK
and EPA) and hand-derived contacts for the pairs those tests do not cover."""
import numpy as np
import pytest

from oracle.zeno_oracle import OracleWorld, gjk_epa, narrow_cpu
from zeno_b200 import scenes

I = (0, 0, 0, 0, 0, 0, 1)  # body at the origin, identity quaternion


def body(x=0.0, y=0.0, z=0.0, q=(0, 0, 0, 1)):
    return (x, y, z, *q)


def sphere(r, at=(0, 0, 0)):
    return (0, *at, r, 0, 0)


def capsule(r, half_len, at=(0, 0, 0)):
    return (1, *at, r, half_len, 0)


def box(hx, hy, hz, at=(0, 0, 0)):
    return (2, *at, hx, hy, hz)


PLANE = (3, 0, 0, 0, 0, 0, 0)


def test_reference_sphere_sphere():  # test_collision.zig:55-69
    r = narrow_cpu(sphere(0.5), I, sphere(0.5), body(0.8))
    assert r is not None
    assert abs(r[2] - 0.2) < 0.01 and abs(r[1][0] - 1.0) < 0.01


def test_reference_sphere_sphere_apart():  # test_collision.zig:71-81
    assert narrow_cpu(sphere(0.5), I, sphere(0.5), body(2.0)) is None


def test_reference_sphere_plane():  # test_collision.zig:173-187
    r = narrow_cpu(sphere(0.5), body(z=0.3), PLANE, I)
    assert r is not None and abs(r[2] - 0.2) < 0.01


def test_reference_sphere_plane_apart():  # test_collision.zig:189-199
    assert narrow_cpu(sphere(0.5), body(z=1.0), PLANE, I) is None


def test_reference_spheres_touching():  # test_collision.zig:219-232
    r = narrow_cpu(sphere(0.5), I, sphere(0.5), body(1.0))
    assert r is None or r[2] <= 0.01


@pytest.mark.parametrize("case,expect", [
    # (geom a, body a, geom b, body b) -> (point, normal, penetration)
    ((capsule(0.1, 0.5), body(z=0.55), PLANE, I), ((0, 0, -0.025), (0, 0, 1), 0.05)),
    ((PLANE, I, capsule(0.1, 0.5), body(z=0.55)), ((0, 0, -0.025), (0, 0, -1), 0.05)),
    ((box(0.5, 0.5, 0.5), body(z=0.4), PLANE, I), ((-0.5, -0.5, -0.1), (0, 0, 1), 0.1)),
    ((sphere(0.3), body(z=0.7), box(0.5, 0.5, 0.5), I), ((0, 0, 0.55), (0, 0, 1), 0.1)),
    ((box(0.5, 0.5, 0.5), I, sphere(0.3), body(z=0.7)), ((0, 0, 0.55), (0, 0, -1), 0.1)),
    ((box(0.5, 0.5, 0.5), I, box(0.5, 0.5, 0.5), body(0.9)), ((0.45, 0, 0), (1, 0, 0), 0.1)),
    ((capsule(0.1, 0.5), I, capsule(0.1, 0.5), body(0.15)), ((0.075, 0, -0.5), (1, 0, 0), 0.05)),
    ((sphere(0.2), body(0.25), capsule(0.1, 0.5), I), ((0.075, 0, 0), (1, 0, 0), 0.05)),
])
def test_hand_derived_pairs(case, expect):
    r = narrow_cpu(*case)
    assert r is not None
    np.testing.assert_allclose(r[0], expect[0], atol=1e-6)
    np.testing.assert_allclose(r[1], expect[1], atol=1e-6)
    assert abs(r[2] - expect[2]) < 1e-6


def test_geoms_placed_by_body_pose():
    """Geom offsets rotate with the body (getWorldCenter), unlike the GPU narrow phase."""
    s = np.sqrt(0.5)
    qz90 = (0, 0, s, s)  # 90 degrees about z: local +x -> world +y
    r = narrow_cpu(sphere(0.5, at=(1.0, 0, 0)), body(q=qz90), sphere(0.5), body(0, 1.8, 0))
    assert r is not None and abs(r[2] - 0.2) < 1e-5
    np.testing.assert_allclose(r[1], (0, 1, 0), atol=1e-5)


@pytest.mark.parametrize("pair", [(capsule(0.1, 0.5), box(0.5, 0.5, 0.5)), (PLANE, PLANE),
                                  ((4, 0, 0, 0, 0.5, 0.5, 0), PLANE)])
def test_pairs_without_a_routine(pair):
    """Box-capsule and plane-plane have no routine; cylinders are not primitives here."""
    assert narrow_cpu(pair[0], I, pair[1], I) is None


def test_extended_mode_adds_pair_types_in_a_rollout():
    """Humanoid (capsule limbs, box feet): over a rollout the reference GPU narrow phase
    never reports a capsule-capsule contact (it has no routine for the pair); the extended
    one does."""
    types = None
    seen = {}
    for mode in (0, 1):
        o = OracleWorld(scenes.humanoid(), num_envs=2, substeps=4, timestep=0.015)
        assert o.set_narrow_phase(mode) == 0
        if types is None:
            geoms = np.frombuffer(o.model_table("geoms"), np.uint32).reshape(-1, 16)
            types = geoms[:, 0]
        acts = np.random.default_rng(3).uniform(-0.4, 0.4, (60, 2, o.num_actuators)).astype(np.float32)
        cc = 0
        for step in range(60):
            o.step(acts[step])
            c = o.state()["contacts"]
            valid = c["position_pen"][..., 3] >= 0
            ga, gb = c["indices"][..., 2], c["indices"][..., 3]
            cc += int((valid & (types[ga] == 1) & (types[gb] == 1)).sum())
        seen[mode] = cc
    assert seen[0] == 0 and seen[1] > 0


# ---- GJK + EPA (narrow-phase mode 2) ----

def test_reference_gjk_sphere_sphere_overlap():  # gjk.zig:712-725
    hit, _ = gjk_epa(sphere(1.0), I, sphere(1.0), body(1.0))
    assert hit


def test_reference_gjk_sphere_sphere_apart():  # gjk.zig:727-740
    assert gjk_epa(sphere(1.0), I, sphere(1.0), body(5.0)) == (False, None)


def test_reference_epa_sphere_sphere_depth():  # gjk.zig:742-762
    hit, res = gjk_epa(sphere(1.0), I, sphere(1.0), body(1.0))
    assert hit and res is not None
    normal, depth = res[0], res[1]
    assert abs(depth - 1.0) <= 0.1
    assert abs(normal[0]) > 0.8


def test_reference_gjk_box_sphere_overlap():  # gjk.zig:764-777
    hit, _ = gjk_epa(box(1.0, 1.0, 1.0), I, sphere(0.5), body(1.2))
    assert hit


def test_reference_gjk_box_sphere_apart():  # gjk.zig:779-792
    hit, _ = gjk_epa(box(1.0, 1.0, 1.0), I, sphere(0.5), body(3.0))
    assert not hit


S45 = float(np.sin(np.pi / 4))


@pytest.mark.parametrize("case,expect", [
    # box half 1 at the origin, upright capsule r .5 beside it at x = 1.3: depth .2 along x
    ((box(1, 1, 1), I, capsule(0.5, 1.0), body(1.3)), ((0.9, 0, 0.5), (1, 0, 0), 0.2)),
    ((capsule(0.5, 1.0), body(1.3), box(1, 1, 1), I), ((0.9, 0, 0.5), (-1, 0, 0), 0.2)),
    # capsule lying along y (90 degrees about x) on top of the box: depth .1 along z
    ((box(1, 1, 1), I, capsule(0.5, 0.8), body(0.2, 0, 1.4, (S45, 0, 0, S45))), ((0.2, 0, 0.95), (0, 0, 1), 0.1)),
])
def test_gjk_box_capsule(case, expect):
    """Mode 2 resolves box-capsule pairs through GJK + EPA: normal from A to B, depth, and
    the midpoint of the witness points, to EPA's tolerance (1e-4)."""
    r = narrow_cpu(*case, mode=2)
    assert r is not None
    np.testing.assert_allclose(r[1], expect[1], atol=1e-4)
    assert abs(r[2] - expect[2]) < 1e-4
    # the contact point lies on the contact normal's line through the overlap; check the
    # coordinate along the normal (the tangential position of EPA's witness is not unique)
    n = np.asarray(expect[1], np.float32)
    assert abs(float(np.dot(r[0], n)) - float(np.dot(expect[0], n))) < 1e-3


def test_gjk_box_capsule_apart():
    assert narrow_cpu(box(1, 1, 1), I, capsule(0.5, 1.0), body(1.6), mode=2) is None


def test_mode2_leaves_other_pairs_as_mode1():
    """Mode 2 changes only box-capsule pairs."""
    cases = [(sphere(0.5), I, sphere(0.5), body(0.8)), (capsule(0.1, 0.5), body(z=0.55), PLANE, I),
             (box(0.5, 0.5, 0.5), I, box(0.5, 0.5, 0.5), body(0.9))]
    for c in cases:
        r1, r2 = narrow_cpu(*c, mode=1), narrow_cpu(*c, mode=2)
        for a, b in zip(r1, r2):
            np.testing.assert_array_equal(a, b)

