"""GPU parity: the sm_100a step (through the C ABI) against the CPU oracle.

Every ABI-visible buffer must match bit for bit -- positions, quaternions, velocities,
angular velocities, accelerations, joint state and torques, observations, rewards,
dones, the 64-byte contact slots and the contact counters -- after 1 step, after 10
steps and over longer rollouts.  Bit-exactness is possible because both sides evaluate
the same canonical single-precision expressions (explicit FMAs, products, Newton-Raphson
reciprocals and reciprocal square roots, the same arctangent polynomial).  How far that
canonical arithmetic lies from the reference kernels' own arithmetic (north_star's 1e-5 /
1e-3 tolerances and the 1000-step energy and contact statistics) is checked against the
oracle's literal arithmetic in test_tolerance_gpu.py."""
import numpy as np
import pytest

from oracle.zeno_oracle import OracleWorld
from parity import CONFIGS, actions, diff_report, make_pair, product_state
from zeno_b200 import ZenoWorld, scenes

pytestmark = pytest.mark.gpu

SCENES = list(CONFIGS)


@pytest.mark.parametrize("name", SCENES)
@pytest.mark.parametrize("nsteps", [1, 10])
def test_rollout_bit_exact(name, nsteps):
    E = 16
    w, o, c = make_pair(name, E)
    rng = np.random.default_rng(1234)
    acts = actions(rng, nsteps, E, w.action_dim, c["act"])
    for s in range(nsteps):
        w.step(acts[s])
        o.step(acts[s])
    bad = diff_report(product_state(w), o.state())
    assert not bad, f"{name} after {nsteps} steps: {bad}"


@pytest.mark.parametrize("name", ["ant", "humanoid", "cartpole"])
def test_long_rollout_and_statistics(name):
    """200 steps bit-exact, and the per-step valid-contact counts equal."""
    E, N = 8, 200
    w, o, c = make_pair(name, E)
    rng = np.random.default_rng(7)
    acts = actions(rng, N, E, w.action_dim, c["act"])
    contacts_p, contacts_o = [], []
    for s in range(N):
        w.step(acts[s])
        o.step(acts[s])
        contacts_p.append((w.get_contacts(zero_copy=False)["position_pen"][..., 3] >= 0).sum())
        contacts_o.append((o.state()["contacts"]["position_pen"][..., 3] >= 0).sum())
    bad = diff_report(product_state(w), o.state())
    assert not bad, f"{name} after {N} steps: {bad}"
    assert contacts_p == contacts_o


def test_multi_env_counts_and_slots_ant():
    """Ant contact bookkeeping: the 64-slot list saturates during step 2 and then freezes,
    while the counter keeps growing (reference behaviour: it is only reset by reset)."""
    E = 4
    w, o, c = make_pair("ant", E)
    rng = np.random.default_rng(3)
    acts = actions(rng, 6, E, w.action_dim, 1.0)
    for s in range(6):
        w.step(acts[s])
        o.step(acts[s])
        assert not diff_report(product_state(w), o.state(), ["contacts", "contact_counts"])
    counts = w.get_contact_counts()
    assert (counts > 64).all()


@pytest.mark.parametrize("name", ["ant", "cartpole", "pendulum_asset"])
def test_step_subset_bit_exact(name):
    E = 8
    w, o, c = make_pair(name, E)
    rng = np.random.default_rng(11)
    acts = actions(rng, 12, E, w.action_dim, c["act"])
    for s in range(12):
        mask = (rng.random(E) < 0.5).astype(np.uint8)
        if s % 4 == 3:
            mask[:] = 1
        w.step_subset(acts[s], mask)
        o.step_subset(acts[s], mask)
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


@pytest.mark.parametrize("name", ["ant", "pendulum_asset"])
def test_reset_and_reset_to_state_bit_exact(name):
    E = 8
    w, o, c = make_pair(name, E)
    rng = np.random.default_rng(5)
    acts = actions(rng, 20, E, w.action_dim, c["act"])
    for s in range(20):
        w.step(acts[s])
        o.step(acts[s])
        if s == 6:
            mask = np.zeros(E, np.uint8)
            mask[[0, 3, 5]] = 1
            w.reset(mask)
            o.reset(mask)
        if s == 12:
            st = product_state(w)
            pos = st["positions"] + rng.uniform(-0.01, 0.01, st["positions"].shape).astype(np.float32)
            mask = (np.arange(E) % 2).astype(np.uint8)
            w.reset_to_state(pos, st["quaternions"], st["velocities"] * 0.5, None, mask)
            o.reset_to_state(pos, st["quaternions"], st["velocities"] * 0.5, None, mask)
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


def test_gravity_timestep_and_substep_override():
    E = 4
    w, o, c = make_pair("ant", E)
    rng = np.random.default_rng(9)
    acts = actions(rng, 9, E, w.action_dim, 1.0)
    for s in range(9):
        if s == 2:
            w.set_gravity((0.0, 0.5, -3.0))
            o.set_gravity((0.0, 0.5, -3.0))
        if s == 4:
            w.set_timestep(0.005)
            o.set_timestep(0.005)
        sub = 0 if s < 6 else 2
        w.step(acts[s], sub)
        o.step(acts[s], sub)
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


def test_extreme_and_nan_actions_bit_exact():
    E = 6
    w, o, c = make_pair("pendulum_asset", E)
    a = np.array([[1e6], [-1e6], [np.nan], [np.inf], [-np.inf], [0.0]], dtype=np.float32)
    for _ in range(3):
        w.step(a)
        o.step(a)
    assert not diff_report(product_state(w), o.state())
    assert np.isfinite(w.get_observations()).all()


@pytest.mark.parametrize("auto_reset", [False, True])
def test_task_extension_bit_exact(auto_reset):
    """Rewards, dones and device-side masked reset with noise (BASELINE Ant episode)."""
    E = 16
    w, o, c = make_pair("ant", E)
    kw = dict(body=1, z_min=0.2, z_max=1.0, auto_reset=auto_reset, noise=0.1, seed=77, env_offset=1000)
    w.set_task(**kw)
    o.set_task(**kw)
    rng = np.random.default_rng(21)
    acts = actions(rng, 60, E, w.action_dim, 1.0)
    saw_done = False
    for s in range(60):
        w.step(acts[s])
        o.step(acts[s])
        st = product_state(w)
        saw_done |= bool(st["dones"].any())
        bad = diff_report(st, o.state())
        assert not bad, f"step {s}: {bad}"
    assert saw_done


@pytest.mark.parametrize("lanes,epb", [(1, 31), (2, 16)])
def test_refilling_lists_bit_exact(lanes, epb):
    """Contact lists refilling after auto-resets, in warps with enough active lanes to
    merge a list cooperatively (70 envs: two full blocks, then a block of 8 or 6 envs that
    sorts serially), every buffer bit-exact at every step."""
    E = 70
    w, o, c = make_pair("ant", E)
    w.set_launch(lanes, epb)
    kw = dict(body=1, z_min=0.2, z_max=1.0, auto_reset=True, noise=0.1, seed=5, env_offset=0)
    w.set_task(**kw)
    o.set_task(**kw)
    rng = np.random.default_rng(33)
    acts = actions(rng, 40, E, w.action_dim, 1.0)
    resets = 0
    for s in range(40):
        w.step(acts[s])
        o.step(acts[s])
        st = product_state(w)
        resets += int(st["dones"].sum())
        bad = diff_report(st, o.state())
        assert not bad, f"step {s}: {bad}"
    assert resets >= 5


@pytest.mark.parametrize("lanes,epb", [(1, 32), (1, 7), (1, 1), (2, 32), (2, 5), (2, 1), (8, 4), (16, 2), (32, 1)])
def test_launch_shapes_agree(lanes, epb):
    """Every launch shape of both kernels computes the same bits: lanes 1, 2 run the
    compressed-state kernel, 8..32 the general kernel."""
    E = 13
    w, o, c = make_pair("ant", E)
    w.set_launch(lanes, epb)
    assert w.get_launch() == (lanes, epb)
    rng = np.random.default_rng(2)
    acts = actions(rng, 5, E, w.action_dim, 1.0)
    for s in range(5):
        w.step(acts[s])
        o.step(acts[s])
    assert not diff_report(product_state(w), o.state())


def test_full_size_ant_sampled_envs_and_determinism():
    """BASELINE size (16384 Ant envs): environments are independent, so a sample of envs
    stepped alone in the oracle must reproduce the batched GPU result bit for bit; a
    second GPU run must reproduce the first (no races)."""
    E, N = 16384, 5
    xml = CONFIGS["ant"]["xml"]()
    from oracle.zeno_oracle import OracleWorld
    from zeno_b200 import ZenoWorld
    rng = np.random.default_rng(0)
    acts = rng.uniform(-1, 1, size=(N, E, 8)).astype(np.float32)
    runs = []
    for _ in range(2):
        w = ZenoWorld(mjcf_string=xml, num_envs=E, substeps=4)
        for s in range(N):
            w.step(acts[s])
        runs.append(product_state(w))
        del w
    assert not diff_report(runs[0], runs[1])
    sample = np.array([0, 1, 777, 4095, 8191, 12000, 16383])
    o = OracleWorld(xml, num_envs=len(sample), substeps=4)
    for s in range(N):
        o.step(acts[s][sample])
    ref = o.state()
    got = {k: v[sample] for k, v in runs[0].items()}
    assert not diff_report(got, ref)


@pytest.mark.parametrize("name", ["ant", "humanoid", "cartpole", "pendulum", "pendulum_asset"])
def test_default_kernel_is_compressed_state(name):
    """Every scene of the parity suite runs on the compressed-state kernel by default."""
    w, _, _ = make_pair(name, 4)
    assert w.get_launch()[0] in (1, 2)


@pytest.mark.parametrize("lanes", [1, 2])
@pytest.mark.parametrize("name", ["humanoid", "cartpole", "pendulum_asset"])
def test_scenes_on_every_lane_count(name, lanes):
    """The compressed-state kernel with 1 and 2 lanes per environment against the oracle."""
    w, o, c = make_pair(name, 6)
    w.set_launch(lanes, 4)
    rng = np.random.default_rng(11)
    acts = actions(rng, 8, 6, w.action_dim, c["act"])
    for s in range(8):
        w.step(acts[s])
        o.step(acts[s])
    assert not diff_report(product_state(w), o.state())


def test_large_scene_uses_general_kernel():
    """A model beyond the constant-bank capacities (64 spheres, 2080 candidate pairs)
    falls back to the general kernel and still matches the oracle bit for bit."""
    xml = scenes.collision_stress(0)
    w = ZenoWorld(mjcf_string=xml, num_envs=3, substeps=2)
    o = OracleWorld(xml, num_envs=3, substeps=2)
    assert w.get_launch()[0] >= 8
    none = np.zeros((3, 0), np.float32)
    for _ in range(3):
        w.step(none)
        o.step(none)
    assert not diff_report(product_state(w), o.state())


@pytest.mark.parametrize("lanes", [1, 2])
def test_hand_over_to_general_kernel(lanes):
    """An environment whose stored contact list the fast kernel cannot represent (a slot
    tuple that is not a broad-phase candidate) is stepped by the general kernel instead;
    the result equals running the general kernel on every environment, and the hand-over
    list is cleared so later steps are unaffected."""
    E = 9
    xml = CONFIGS["ant"]["xml"]()
    rng = np.random.default_rng(5)
    acts = actions(rng, 6, E, 8, 1.0)
    runs = []
    for ln, epb in ((lanes, 32), (8, 4)):
        w = ZenoWorld(mjcf_string=xml, num_envs=E, substeps=4)
        w.set_launch(ln, epb)
        for s in range(3):
            w.step(acts[s])
        c = w.get_contacts()  # zero-copy view of the contact buffer
        c["indices"][4, 0] = (1, 1, 1, 1)  # geom 1 with itself: not a candidate pair
        for s in range(3, 6):
            w.step(acts[s])
        runs.append(product_state(w))
    assert not diff_report(runs[0], runs[1])


@pytest.mark.parametrize("name,lanes,mode", [("ant", 1, 1), ("ant", 2, 1), ("ant", 8, 1), ("cartpole", 1, 1),
                                             ("pendulum_asset", 1, 1), ("humanoid", None, 1), ("ant", 1, 2),
                                             ("humanoid", None, 2)])
def test_extended_narrow_phase_bit_exact(name, lanes, mode):
    """Narrow phases 1 (the reference's CPU detectCollision: sphere/capsule/box/plane pairs,
    geoms placed by body pose) and 2 (the same plus GJK + EPA for box-capsule pairs) on
    both kernels against the oracle.  Humanoid has more hittable candidates in these modes
    than the compressed-state kernel holds (64), so it runs on the general kernel; Ant has
    no box, so mode 2 keeps it on the compressed-state kernel."""
    E = 6
    w, o, c = make_pair(name, E)
    w.set_narrow_phase(mode)
    assert o.set_narrow_phase(mode) == 0
    if lanes is not None:
        w.set_launch(lanes, 4)
    elif name == "humanoid":
        assert w.get_launch()[0] >= 8
    rng = np.random.default_rng(21)
    acts = actions(rng, 12, E, w.action_dim, c["act"])
    for s in range(12):
        w.step(acts[s])
        o.step(acts[s])
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


def test_extended_narrow_phase_drop_scene():
    """The 64-body drop scene (spheres, capsules, boxes on a plane; general kernel) with
    the extended narrow phase, where every pair type the reference CPU code handles occurs."""
    xml = scenes.collision_stress(0)
    kw = dict(num_envs=2, substeps=2, max_contacts_per_env=256)
    w, o = ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw)
    w.set_narrow_phase(1)
    o.set_narrow_phase(1)
    none = np.zeros((2, 0), np.float32)
    for s in range(20):
        w.step(none)
        o.step(none)
    st = product_state(w)
    assert not diff_report(st, o.state())
    assert (st["contacts"]["position_pen"][..., 3] >= 0).sum() > 0


BOX_CAPSULE = """<mujoco model="box_capsule">
  <option timestep="0.005" gravity="0 0 -9.81"/>
  <worldbody>
    <geom type="plane" size="5 5 0.1" friction="0.8 0.005 0.0001"/>
    <body name="crate" pos="0 0 0.1">
      <joint type="free"/>
      <geom type="box" size="0.3 0.3 0.1" density="500"/>
    </body>
    <body name="log" pos="0.05 0.02 0.24" quat="0.7071068 0.7071068 0 0">
      <joint type="free"/>
      <geom type="capsule" size="0.05 0.2" density="800"/>
    </body>
    <body name="post" pos="-0.15 0.1 0.45" quat="0.9961947 0 0.0871557 0">
      <joint type="free"/>
      <geom type="capsule" size="0.04 0.2" density="800"/>
    </body>
    <body name="crate2" pos="0.9 0 0.35" quat="0.9659258 0.2588190 0 0">
      <joint type="free"/>
      <geom type="box" size="0.1 0.2 0.1" density="500"/>
    </body>
    <body name="rod" pos="0.9 0.05 0.08" quat="0.7071068 0 0.7071068 0">
      <joint type="free"/>
      <geom type="capsule" size="0.06 0.25" density="800"/>
    </body>
  </worldbody>
</mujoco>
"""


SHARED_KEYS = """<mujoco model="shared_keys">
  <option timestep="0.01" gravity="0 0 -9.81"/>
  <worldbody>
    <geom name="floor" type="plane" size="5 5 0.1"/>
    <body name="bell" pos="0 0 0.6">
      <freejoint/>
      <geom type="sphere" size="0.1" pos="-0.2 0 0"/>
      <geom type="sphere" size="0.1" pos="0.2 0 0.05"/>
    </body>
    <body name="hammer" pos="0.3 0 0.9">
      <freejoint/>
      <geom type="sphere" size="0.12" pos="0 0 -0.15"/>
      <geom type="capsule" size="0.05 0.15" pos="0 0 0.1"/>
    </body>
  </worldbody>
</mujoco>"""


@pytest.mark.parametrize("lanes,epb", [(1, 31), (2, 16)])
@pytest.mark.parametrize("mode", [0, 1])
def test_shared_key_pairs_bit_exact(lanes, epb, mode):
    """Two hittable pairs on one body pair (each body's two geoms against the plane and
    against each other): the warm-start match of one pair reads the other's previous
    point, so the compressed-state kernel runs its narrow phase in two passes.  Bit-exact
    against the oracle while the bodies drop, land, tip and settle (40 envs: full warps,
    so refilling lists are merged cooperatively)."""
    E = 40
    kw = dict(num_envs=E, substeps=4, max_contacts_per_env=32)
    w, o = ZenoWorld(mjcf_string=SHARED_KEYS, **kw), OracleWorld(SHARED_KEYS, **kw)
    w.set_narrow_phase(mode)
    assert o.set_narrow_phase(mode) == 0
    w.set_launch(lanes, epb)
    assert w.get_launch() == (lanes, epb)
    rng = np.random.default_rng(8)
    st0 = product_state(w)
    pos, quat = st0["positions"].copy(), st0["quaternions"].copy()
    pos[:, 1:, :3] += rng.uniform(-0.05, 0.05, size=(E, pos.shape[1] - 1, 3)).astype(np.float32)
    w.reset_to_state(pos, quat)
    o.reset_to_state(pos, quat)
    none = np.zeros((E, 0), np.float32)
    hits = 0
    for s in range(60):
        w.step(none)
        o.step(none)
        st = product_state(w)
        bad = diff_report(st, o.state())
        assert not bad, f"step {s}: {bad}"
        hits += int((st["contacts"]["position_pen"][..., 3] >= 0).sum())
    assert hits > 0


@pytest.mark.parametrize("lanes", [8, 32])
def test_gjk_box_capsule_scene(lanes):
    """Capsules resting on and under boxes: with narrow phase 2 the box-capsule pairs go
    through GJK + EPA on the GPU and agree with the oracle bit for bit; mode 1 reports no
    contact for them (no routine), mode 2 does."""
    E = 4
    kw = dict(num_envs=E, substeps=4, max_contacts_per_env=32)
    w, o = ZenoWorld(mjcf_string=BOX_CAPSULE, **kw), OracleWorld(BOX_CAPSULE, **kw)
    w.set_narrow_phase(2)
    assert o.set_narrow_phase(2) == 0
    w.set_launch(lanes, 1)
    geoms = np.frombuffer(o.model_table("geoms"), np.uint32).reshape(-1, 16)
    types = geoms[:, 0]
    none = np.zeros((E, 0), np.float32)
    gjk_hits = 0
    for s in range(40):
        w.step(none)
        o.step(none)
        st = product_state(w)
        bad = diff_report(st, o.state())
        assert not bad, f"step {s}: {bad}"
        c = st["contacts"]
        valid = c["position_pen"][..., 3] >= 0
        ta, tb = types[c["indices"][..., 2]], types[c["indices"][..., 3]]
        gjk_hits += int((valid & (((ta == 1) & (tb == 2)) | ((ta == 2) & (tb == 1)))).sum())
    assert gjk_hits > 0


def test_general_blocking_follows_the_narrow_phase():
    """The general kernel takes 16 environments per block when GJK + EPA can run (narrow
    phase 2 with box-capsule candidates) and 4 otherwise; a shape set by the caller is
    kept; results are the oracle's either way."""
    E = 40
    w, o, c = make_pair("humanoid", E)
    acts = actions(np.random.default_rng(21), 6, E, w.action_dim, c["act"])
    for mode, shape in ((2, (8, 16)), (1, (8, 4)), (2, (8, 16))):
        w.set_narrow_phase(mode)
        assert o.set_narrow_phase(mode) == 0
        assert w.get_launch() == shape
        for s in range(2):
            w.step(acts[s])
            o.step(acts[s])
        assert not diff_report(product_state(w), o.state())
    w.set_launch(8, 2)
    w.set_narrow_phase(1)
    w.set_narrow_phase(2)
    assert w.get_launch() == (8, 2)


def test_extended_narrow_phase_drop_scene_gjk():
    """The 64-body drop scene with narrow phase 2 (box-capsule through GJK + EPA)."""
    xml = scenes.collision_stress(0)
    kw = dict(num_envs=2, substeps=2, max_contacts_per_env=256)
    w, o = ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw)
    w.set_narrow_phase(2)
    o.set_narrow_phase(2)
    none = np.zeros((2, 0), np.float32)
    for s in range(20):
        w.step(none)
        o.step(none)
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


def test_narrow_phase_switch_mid_run():
    """Switching the narrow phase between steps re-packs the compressed model; the oracle
    switched at the same steps agrees."""
    E = 5
    w, o, c = make_pair("humanoid", E)
    rng = np.random.default_rng(4)
    acts = actions(rng, 15, E, w.action_dim, c["act"])
    for s in range(15):
        mode = 1 if 5 <= s < 10 else 0
        w.set_narrow_phase(mode)
        o.set_narrow_phase(mode)
        assert w.get_narrow_phase() == mode
        w.step(acts[s])
        o.step(acts[s])
    assert not diff_report(product_state(w), o.state())


# ---- corrected semantics (general kernel) ----

@pytest.mark.parametrize("name,lanes", [("ant", 8), ("ant", 32), ("humanoid", 16), ("cartpole", 8),
                                        ("pendulum_asset", 8), ("pendulum", 32)])
def test_corrected_semantics_bit_exact(name, lanes):
    """Corrected semantics (MJCF compiler rules, rotated geom frames and bounds, the list
    rebuilt every substep, B->A normals, narrow phase 2) on the general kernel against the
    oracle, bit for bit."""
    E = 5
    w, o, c = make_pair(name, E, semantics="corrected")
    assert w.get_narrow_phase() == 2
    assert w.get_launch()[0] >= 8  # corrected worlds run on the general kernel
    w.set_launch(lanes, 1)
    rng = np.random.default_rng(17)
    acts = actions(rng, 15, E, w.action_dim, c["act"])
    for s in range(15):
        w.step(acts[s])
        o.step(acts[s])
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


def test_corrected_semantics_scenes():
    """The box-capsule scene and the 64-body drop scene under corrected semantics, with a
    narrow-phase switch to mode 1 and back; mode 0 is refused."""
    for xml, E, M in ((BOX_CAPSULE, 3, 32), (scenes.collision_stress(1), 2, 256)):
        kw = dict(num_envs=E, substeps=4, max_contacts_per_env=M, semantics="corrected")
        w, o = ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw)
        with pytest.raises(RuntimeError):
            w.set_narrow_phase(0)
        none = np.zeros((E, 0), np.float32)
        for s in range(24):
            mode = 1 if 8 <= s < 16 else 2
            w.set_narrow_phase(mode)
            assert o.set_narrow_phase(mode) == 0
            w.step(none)
            o.step(none)
            bad = diff_report(product_state(w), o.state())
            assert not bad, f"step {s}: {bad}"


def test_corrected_resting_contact_on_gpu():
    """Touching bodies stay at rest under corrected semantics on the GPU as in the oracle."""
    xml = ('<mujoco><option timestep="0.005"/><worldbody><geom type="plane" size="5 5 .1"/>'
           '<body pos="0 0 0.1"><joint type="free"/><geom type="box" size="0.1 0.1 0.1"/></body>'
           '<body pos="0 0 0.3"><joint type="free"/><geom type="sphere" size="0.1"/></body>'
           '<body pos="0.5 0 0.05" euler="0 90 0"><joint type="free"/><geom type="capsule" size="0.05 0.2"/></body>'
           '</worldbody></mujoco>')
    kw = dict(num_envs=4, substeps=8, max_contacts_per_env=32, semantics="corrected")
    w, o = ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw)
    none = np.zeros((4, 0), np.float32)
    for _ in range(100):
        w.step(none)
        o.step(none)
    st = product_state(w)
    assert not diff_report(st, o.state())
    assert np.abs(st["velocities"][:, 1:, :3]).max() < 0.05



# ---- grid broad phase (same slots as the all-candidate-pairs sweep) ----

@pytest.mark.parametrize("name,mode,sem", [("ant", 0, "reference"), ("humanoid", 1, "reference"),
                                           ("cartpole", 0, "reference"), ("ant", 2, "corrected"),
                                           ("humanoid", 2, "corrected")])
def test_grid_broad_phase_bit_exact(name, mode, sem):
    """The general kernel with the hashed grid forced (broad phase 2) against the oracle's
    all-pairs sweep, bit for bit."""
    E = 4
    w, o, c = make_pair(name, E, semantics=sem)
    w.set_launch(8, 4)
    w.set_narrow_phase(mode)
    assert o.set_narrow_phase(mode) == 0
    w.set_broad_phase(2)
    assert w.get_broad_phase() == 2
    rng = np.random.default_rng(23)
    acts = actions(rng, 12, E, w.action_dim, c["act"])
    for s in range(12):
        w.step(acts[s])
        o.step(acts[s])
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


@pytest.mark.parametrize("sem", ["reference", "corrected"])
def test_grid_drop_scene(sem):
    xml = scenes.collision_stress(2)
    kw = dict(num_envs=2, substeps=4, max_contacts_per_env=256, semantics=sem)
    w, o = ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw)
    w.set_narrow_phase(1)
    o.set_narrow_phase(1)
    w.set_broad_phase(2)
    none = np.zeros((2, 0), np.float32)
    for s in range(15):
        w.step(none)
        o.step(none)
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"


@pytest.mark.parametrize("sem", ["reference", "corrected"])
def test_large_scene_uses_the_grid(sem):
    """601 geoms (past the reference's 512-geom switch to its spatial hash): the default
    broad phase is the grid; its slots equal the oracle's all-pairs sweep and the general
    kernel's own sweep (broad phase 1)."""
    xml = scenes.sphere_pile(0)
    kw = dict(num_envs=2, substeps=4, max_contacts_per_env=1024, semantics=sem)
    o = OracleWorld(xml, **kw)
    if sem == "corrected":
        o.set_narrow_phase(1)
    runs = []
    for bp in (0, 1):
        w = ZenoWorld(mjcf_string=xml, **kw)
        assert w.get_launch() == (32, 1)  # one warp per (large) environment
        if sem == "corrected":
            w.set_narrow_phase(1)
        w.set_broad_phase(bp)
        runs.append(w)
    none = np.zeros((2, 0), np.float32)
    for s in range(12):
        for w in runs:
            w.step(none)
        o.step(none)
        ref = o.state()
        for w in runs:
            bad = diff_report(product_state(w), ref)
            assert not bad, f"step {s}, broad phase {w.get_broad_phase()}: {bad}"
    assert product_state(runs[0])["contact_counts"].min() > 600


def test_grid_falls_back_off_grid():
    """A geom centre more than 500 cells from the origin sends that environment through
    the all-pairs sweep for the substep; results stay identical to the oracle's."""
    xml = ('<mujoco><option timestep="0.005"/><worldbody><geom type="plane" size="5 5 .1"/>'
           '<body pos="0 0 0.3"><joint type="free"/><geom type="sphere" size="0.1"/></body>'
           '<body pos="0.15 0 0.3"><joint type="free"/><geom type="sphere" size="0.1"/></body>'
           '<body pos="0 0 0.55"><joint type="free"/><geom type="box" size="0.1 0.1 0.1"/></body>'
           '<body pos="500 0 0.3"><joint type="free"/><geom type="sphere" size="0.1"/></body>'
           '</worldbody></mujoco>')
    kw = dict(num_envs=3, substeps=4, max_contacts_per_env=32)
    w, o = ZenoWorld(mjcf_string=xml, **kw), OracleWorld(xml, **kw)
    w.set_launch(8, 4)
    w.set_narrow_phase(1)
    o.set_narrow_phase(1)
    w.set_broad_phase(2)
    none = np.zeros((3, 0), np.float32)
    for s in range(10):
        w.step(none)
        o.step(none)
        bad = diff_report(product_state(w), o.state())
        assert not bad, f"step {s}: {bad}"
