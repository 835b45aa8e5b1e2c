"""MJCF descriptions of the benchmark workloads.

``ant()`` and ``humanoid()`` describe the same robots as the reference's shipped
``assets/ant.xml`` and ``assets/humanoid.xml`` (identical bodies, joints, geoms, actuator
gears, defaults and sensors; colours and comments dropped), because the benchmark runs
the reference Ant.  ``pendulum()`` and ``cartpole()`` build the synthetic variants the
benchmark configuration describes in words (3 bodies each), and ``collision_stress()``
generates the seeded 64-body drop scene.  ``pendulum_asset()`` mirrors the reference's
pendulum test fixture (tests/test_python_integration.py PENDULUM_MJCF), which the API
tests use.

All functions return MJCF text accepted by ``zeno_world_create_from_string``.
"""
from __future__ import annotations

import numpy as np


def ant() -> str:
    """Ant: torso sphere + 4 two-segment capsule legs, free root, 8 limited hinges."""
    legs = [
        # (leg body, hip name, hip pos, hip capsule end, foot pos, ankle axis, foot capsule end)
        ("front_right", "1", (0.2, 0.2), (0.2, 0.2), (0.2, 0.2), "-1 1 0", (0.4, 0.4)),
        ("front_left", "2", (-0.2, 0.2), (-0.2, 0.2), (-0.2, 0.2), "1 1 0", (-0.4, 0.4)),
        ("back_right", "3", (0.2, -0.2), (0.2, -0.2), (0.2, -0.2), "-1 -1 0", (0.4, -0.4)),
        ("back_left", "4", (-0.2, -0.2), (-0.2, -0.2), (-0.2, -0.2), "1 -1 0", (-0.4, -0.4)),
    ]
    body = []
    for name, k, hp, he, fp, ax, fe in legs:
        body.append(
            f'''      <body name="{name}_leg" pos="{hp[0]} {hp[1]} 0">
        <joint name="hip_{k}" type="hinge" axis="0 0 1" range="-30 30"/>
        <geom type="capsule" fromto="0 0 0 {he[0]} {he[1]} 0" size="0.08"/>
        <body name="{name}_foot" pos="{fp[0]} {fp[1]} 0">
          <joint name="ankle_{k}" type="hinge" axis="{ax}" range="-70 -30"/>
          <geom type="capsule" fromto="0 0 0 {fe[0]} {fe[1]} 0" size="0.08"/>
        </body>
      </body>''')
    motors = "\n".join(
        f'    <motor joint="{j}_{k}" ctrlrange="-1 1" gear="150"/>'
        for k in "1234" for j in ("hip", "ankle"))
    jp = "\n".join(f'    <jointpos joint="{j}_{k}"/>' for k in "1234" for j in ("hip", "ankle"))
    jv = "\n".join(f'    <jointvel joint="{j}_{k}"/>' for k in "1234" for j in ("hip", "ankle"))
    return f'''<mujoco model="ant">
  <option timestep="0.01" gravity="0 0 -9.81"/>
  <default>
    <joint armature="1" damping="1" limited="true"/>
    <geom contype="1" conaffinity="1" condim="3" friction="1 0.5 0.5" density="5" margin="0.01"/>
  </default>
  <worldbody>
    <geom type="plane" size="40 40 0.1"/>
    <body name="torso" pos="0 0 0.75">
      <joint name="root" type="free"/>
      <geom name="torso_geom" type="sphere" size="0.25"/>
{chr(10).join(body)}
    </body>
  </worldbody>
  <actuator>
{motors}
  </actuator>
  <sensor>
    <framepos objtype="body" objname="torso"/>
    <framequat objtype="body" objname="torso"/>
    <framelinvel objtype="body" objname="torso"/>
    <frameangvel objtype="body" objname="torso"/>
{jp}
{jv}
  </sensor>
</mujoco>
'''


def humanoid() -> str:
    """Humanoid: capsule limbs, sphere head, box feet, free root, 13 limited hinges."""
    def limb(name, pos, jname, axis, rng, geom, inner="", ind="      "):
        return (f'{ind}<body name="{name}" pos="{pos}">\n'
                f'{ind}  <joint name="{jname}" type="hinge" axis="{axis}" range="{rng}"/>\n'
                f'{ind}  {geom}\n{inner}{ind}</body>\n')

    cap = lambda ft, r: f'<geom type="capsule" fromto="{ft}" size="{r}"/>'
    foot = '<geom type="box" size="0.05 0.03 0.08" pos="0.03 0 0"/>'
    i3, i4, i5 = " " * 10, " " * 12, " " * 14

    def arm(side, sx, sh_rng):
        lower = limb(f"{side}_lower_arm", f"{sx} 0 0", f"{side}_elbow", "0 1 0", "-90 50",
                     cap(f"0 0 0 {sx} 0 0", "0.035"), ind=i5)
        return limb(f"{side}_upper_arm", f"{sx} 0 0.12", f"{side}_shoulder_x", "1 0 0", sh_rng,
                    cap(f"0 0 0 {sx} 0 0", "0.04"), lower, ind=i4)

    def leg(side, x):
        f = limb(f"{side}_foot", "0 0 -0.3", f"{side}_ankle", "0 1 0", "-50 50", foot, ind=i4)
        shin = limb(f"{side}_shin", "0 0 -0.34", f"{side}_knee", "0 1 0", "-160 -2",
                    cap("0 0 0 0 0 -0.3", "0.05"), f, ind=i3)
        return limb(f"{side}_thigh", f"{x} 0 -0.05", f"{side}_hip_x", "1 0 0", "-25 110",
                    cap("0 0 0 0 0 -0.34", "0.06"), shin, ind=" " * 6)

    head = limb("head", "0 0 0.25", "neck", "0 1 0", "-40 40",
                '<geom name="head_geom" type="sphere" size="0.1" pos="0 0 0.1"/>', ind=i4)
    upper = limb("upper_torso", "0 0 0.25", "abdomen_x", "1 0 0", "-35 35",
                 '<geom name="upper_torso_geom" type="capsule" fromto="0 0 0 0 0 0.15" size="0.1"/>',
                 head + arm("right", -0.18, "-85 60") + arm("left", 0.18, "-60 85"), ind=i3)
    torso = limb("torso", "0 0 0.2", "abdomen_y", "0 1 0", "-45 45",
                 '<geom name="torso_geom" type="capsule" fromto="0 0 0 0 0 0.25" size="0.1"/>', upper,
                 ind=" " * 6)
    joints = ["abdomen_y", "abdomen_x", "neck", "right_shoulder_x", "right_elbow", "left_shoulder_x",
              "left_elbow", "right_hip_x", "right_knee", "right_ankle", "left_hip_x", "left_knee",
              "left_ankle"]
    gears = [100, 100, 25, 75, 75, 75, 75, 150, 150, 90, 150, 150, 90]
    motors = "\n".join(f'    <motor joint="{j}" ctrlrange="-1 1" gear="{g}"/>' for j, g in zip(joints, gears))
    jp = "\n".join(f'    <jointpos joint="{j}"/>' for j in joints)
    jv = "\n".join(f'    <jointvel joint="{j}"/>' for j in joints)
    return f'''<mujoco model="humanoid">
  <option timestep="0.005" gravity="0 0 -9.81"/>
  <default>
    <joint armature="0.01" damping="0.5" limited="true"/>
    <geom contype="1" conaffinity="1" condim="3" friction="0.8 0.1 0.1" margin="0.001"/>
  </default>
  <worldbody>
    <geom type="plane" size="50 50 0.1"/>
    <body name="pelvis" pos="0 0 1.25">
      <joint name="root" type="free"/>
      <geom name="pelvis_geom" type="capsule" fromto="-0.1 0 0 0.1 0 0" size="0.08"/>
{torso}{leg("right", -0.1)}{leg("left", 0.1)}    </body>
  </worldbody>
  <actuator>
{motors}
  </actuator>
  <sensor>
    <framepos objtype="body" objname="pelvis"/>
    <framequat objtype="body" objname="pelvis"/>
    <framelinvel objtype="body" objname="pelvis"/>
    <frameangvel objtype="body" objname="pelvis"/>
{jp}
{jv}
  </sensor>
</mujoco>
'''


def pendulum() -> str:
    """Synthetic pendulum: world + welded base + 1 m capsule pole (r 0.05, density 1000),
    hinge about y, motor gear 1, ctrl [-1, 1], dt 0.01, no plane (no contacts)."""
    return '''<mujoco model="pendulum_b">
  <option timestep="0.01" gravity="0 0 -9.81"/>
  <worldbody>
    <body name="base" pos="0 0 2">
      <geom type="sphere" size="0.05" contype="0" conaffinity="0"/>
      <body name="pole" pos="0 0 0">
        <joint name="hinge" type="hinge" axis="0 1 0"/>
        <geom type="capsule" fromto="0 0 0 0 0 -1" size="0.05" density="1000" contype="0" conaffinity="0"/>
      </body>
    </body>
  </worldbody>
  <actuator>
    <motor joint="hinge" ctrlrange="-1 1" gear="1"/>
  </actuator>
  <sensor>
    <jointpos joint="hinge"/>
    <jointvel joint="hinge"/>
  </sensor>
</mujoco>
'''


def cartpole() -> str:
    """Synthetic cartpole: cart box 0.2x0.1x0.1 on a slider (range +-1 m, gear 100),
    pole capsule 0.045 x 0.6 m on a hinge about y, ground plane, dt 0.01."""
    return '''<mujoco model="cartpole_b">
  <option timestep="0.01" gravity="0 0 -9.81"/>
  <worldbody>
    <geom type="plane" size="10 10 0.1"/>
    <geom type="box" pos="0 0 0.05" size="10 0.05 0.05" contype="0" conaffinity="0"/>
    <body name="cart" pos="0 0 0.15">
      <joint name="slider" type="slide" axis="1 0 0" range="-1 1"/>
      <geom type="box" size="0.1 0.05 0.05" mass="1"/>
      <body name="pole" pos="0 0 0.05">
        <joint name="hinge" type="hinge" axis="0 1 0"/>
        <geom type="capsule" fromto="0 0 0 0 0 0.6" size="0.045" mass="0.1"/>
      </body>
    </body>
  </worldbody>
  <actuator>
    <motor joint="slider" ctrlrange="-1 1" gear="100"/>
  </actuator>
  <sensor>
    <jointpos joint="slider"/>
    <jointvel joint="slider"/>
    <jointpos joint="hinge"/>
    <jointvel joint="hinge"/>
  </sensor>
</mujoco>
'''


def pendulum_asset() -> str:
    """Pendulum with base sphere, pole capsule, bob sphere and a ground plane (the
    reference's test fixture model; 4 bodies, contacts against the plane)."""
    return '''<mujoco model="test_pendulum">
  <option timestep="0.02" gravity="0 0 -9.81"/>
  <worldbody>
    <geom type="plane" size="5 5 0.1"/>
    <body name="base" pos="0 0 1.5">
      <geom type="sphere" size="0.05" mass="0"/>
      <body name="pole" pos="0 0 0">
        <joint name="hinge" type="hinge" axis="0 1 0" damping="0.1"/>
        <geom type="capsule" fromto="0 0 0 0 0 -1" size="0.02" mass="1"/>
        <body name="bob" pos="0 0 -1">
          <geom type="sphere" size="0.1" mass="1"/>
        </body>
      </body>
    </body>
  </worldbody>
  <actuator>
    <motor joint="hinge" ctrlrange="-5 5" gear="1"/>
  </actuator>
  <sensor>
    <jointpos joint="hinge"/>
    <jointvel joint="hinge"/>
  </sensor>
</mujoco>
'''


def collision_stress(seed: int = 0, n_spheres: int = 32, n_capsules: int = 16, n_boxes: int = 16) -> str:
    """Seeded drop scene: free spheres r~U(.05,.15), capsules r .05 x len U(.1,.3), boxes with
    half-extents U(.05,.15), density 1000, friction 0.8, uniform poses in a 2 m cube 0.5 m
    above a ground plane; dt 0.005."""
    rng = np.random.default_rng(seed)
    bodies = []
    k = 0

    def pose():
        p = rng.uniform([-1, -1, 0.5], [1, 1, 2.5])
        q = rng.normal(size=4)
        q /= np.linalg.norm(q)
        return p, q

    fr = 'friction="0.8 0.005 0.0001" density="1000"'
    for _ in range(n_spheres):
        p, q = pose()
        r = rng.uniform(0.05, 0.15)
        bodies.append((p, q, f'<geom type="sphere" size="{r:.6f}" {fr}/>'))
    for _ in range(n_capsules):
        p, q = pose()
        hl = 0.5 * rng.uniform(0.1, 0.3)
        bodies.append((p, q, f'<geom type="capsule" size="0.05 {hl:.6f}" {fr}/>'))
    for _ in range(n_boxes):
        p, q = pose()
        h = rng.uniform(0.05, 0.15, size=3)
        bodies.append((p, q, f'<geom type="box" size="{h[0]:.6f} {h[1]:.6f} {h[2]:.6f}" {fr}/>'))
    parts = []
    for p, q, g in bodies:
        k += 1
        parts.append(
            f'    <body name="b{k}" pos="{p[0]:.6f} {p[1]:.6f} {p[2]:.6f}" '
            f'quat="{q[0]:.6f} {q[1]:.6f} {q[2]:.6f} {q[3]:.6f}">\n'
            f'      <joint type="free"/>\n      {g}\n    </body>')
    return ('<mujoco model="collision_stress">\n  <option timestep="0.005" gravity="0 0 -9.81"/>\n'
            '  <worldbody>\n    <geom type="plane" size="20 20 0.1" friction="0.8 0.005 0.0001"/>\n'
            + "\n".join(parts) + '\n  </worldbody>\n</mujoco>\n')


def sphere_pile(seed: int = 0, n: int = 600, extent: float = 1.5, height: float = 1.0) -> str:
    """Seeded large scene past the reference's spatial-hash threshold (more than 512 geoms):
    n free spheres r~U(.03,.06) on a jittered lattice over a 2*extent square, stacked from
    0.1 m to `height`, a few overlapping their neighbours, above a ground plane; dt 0.005."""
    rng = np.random.default_rng(seed)
    side = int(np.ceil(np.sqrt(n / 4)))
    layers = int(np.ceil(n / (side * side)))
    parts = []
    k = 0
    for i in range(side):
        for j in range(side):
            for h in range(layers):
                if k >= n:
                    break
                x = -extent + (i + 0.5) * 2 * extent / side + rng.uniform(-0.02, 0.02)
                y = -extent + (j + 0.5) * 2 * extent / side + rng.uniform(-0.02, 0.02)
                z = 0.1 + h * (height - 0.1) / max(layers - 1, 1) + rng.uniform(-0.02, 0.02)
                r = rng.uniform(0.03, 0.06)
                k += 1
                parts.append(f'    <body name="s{k}" pos="{x:.6f} {y:.6f} {z:.6f}">\n      <joint type="free"/>\n'
                             f'      <geom type="sphere" size="{r:.6f}" friction="0.8 0.005 0.0001"/>\n    </body>')
    return ('<mujoco model="sphere_pile">\n  <option timestep="0.005" gravity="0 0 -9.81"/>\n'
            '  <worldbody>\n    <geom type="plane" size="20 20 0.1" friction="0.8 0.005 0.0001"/>\n'
            + "\n".join(parts) + '\n  </worldbody>\n</mujoco>\n')


BY_NAME = {
    "ant": ant,
    "humanoid": humanoid,
    "pendulum": pendulum,
    "cartpole": cartpole,
    "pendulum_asset": pendulum_asset,
    "collision_stress": collision_stress,
}
