"""The behavioural checks of the reference's Python integration suite
(tests/test_python_integration.py in Lulzx/zeno), run against zeno_b200's ZenoWorld /
ZenoEnv on the GPU: lifecycle, shapes and dtypes, zero-copy identity and in-place
updates, 1024-env batching, subset stepping, masked reset, extreme/NaN actions, state
round trip, gravity and timestep mutation, accelerations, sensors and profiling."""
import numpy as np
import pytest

import zeno_b200
from zeno_b200 import ZenoEnv, ZenoWorld, scenes

pytestmark = pytest.mark.gpu
PEND = scenes.pendulum_asset()


def world(n=1, **kw):
    return ZenoWorld(mjcf_string=PEND, num_envs=n, **kw)


def test_lifecycle_and_dims():
    w = world()
    assert w.num_envs == 1 and w.obs_dim > 0 and w.action_dim > 0
    with pytest.raises(ValueError):
        ZenoWorld()
    w.reset()
    w.step(np.zeros((1, w.action_dim), np.float32))
    obs = w.get_observations()
    assert obs.shape == (1, w.obs_dim) and obs.dtype == np.float32
    for _ in range(100):
        w.step(np.zeros((1, w.action_dim), np.float32))
    assert np.isfinite(w.get_observations()).all()
    info = world(4).get_info()
    assert info["num_envs"] == 4 and info["num_bodies"] > 0 and info["timestep"] > 0
    assert isinstance(zeno_b200.version(), str) and zeno_b200.is_metal_available() is True


def test_zero_copy_semantics():
    w = world(2)
    w.reset()
    p1, p2 = w.get_body_positions(zero_copy=True), w.get_body_positions(zero_copy=True)
    assert p1.ctypes.data == p2.ctypes.data
    cp = w.get_body_positions(zero_copy=False)
    assert cp.ctypes.data != p1.ctypes.data
    np.testing.assert_array_equal(cp, p1)
    snap = p1.copy()
    for _ in range(10):
        w.step(np.ones((2, w.action_dim), np.float32))
    assert not np.array_equal(p1, snap)  # the view reflects the GPU's writes in place
    o1, o2 = w.get_observations(), w.get_observations()
    assert o1.ctypes.data != o2.ctypes.data


def test_host_writes_through_views_reach_the_gpu():
    ball = ('<mujoco><option timestep="0.01" gravity="0 0 0"/><worldbody><body name="b" pos="0 0 1">'
            '<joint type="free"/><geom type="sphere" size="0.1"/></body></worldbody></mujoco>')
    w = ZenoWorld(mjcf_string=ball, num_envs=2)
    pos = w.get_body_positions(zero_copy=True)
    vel = w.get_body_velocities(zero_copy=True)
    pos[1, 1, 2] += 0.5  # lift the ball of env 1 through the zero-copy view
    vel[0, 1, 0] = 2.0   # push the ball of env 0
    w.step(np.zeros((2, 0), np.float32))
    after = w.get_body_positions(zero_copy=False)
    assert after[1, 1, 2] == pytest.approx(1.5, abs=1e-5)
    assert after[0, 1, 0] == pytest.approx(2.0 * 0.999 * 0.01, rel=1e-4)


def test_shapes():
    n = 4
    w = world(n)
    w.reset()
    nb, nj = w.num_bodies, w.num_joints
    for arr in (w.get_body_positions(), w.get_body_quaternions(), w.get_body_velocities(),
                w.get_body_angular_velocities()):
        assert arr.shape == (n, nb, 4) and arr.dtype == np.float32
    assert w.get_joint_positions().shape == (n, nj)
    assert w.get_joint_velocities().shape == (n, nj)
    assert w.get_contacts().shape == (n, w.max_contacts_per_env)
    assert w.get_contact_counts().shape == (n,)


def test_batched_1024():
    n = 1024
    w = world(n)
    w.reset()
    assert w.get_observations().shape == (n, w.obs_dim)
    assert w.get_rewards().shape == (n,) and w.get_dones().shape == (n,)
    w.step(np.random.uniform(-1, 1, (n, w.action_dim)).astype(np.float32))
    assert np.isfinite(w.get_observations()).all()
    env = ZenoEnv(mjcf_string=PEND, num_envs=n)
    obs = env.reset()
    assert obs.shape == (n, env.observation_dim)
    obs, r, d, info = env.step(np.random.uniform(-1, 1, (n, env.action_dim)).astype(np.float32))
    assert obs.shape == (n, env.observation_dim) and r.shape == (n,) and d.shape == (n,)


def test_step_subset_leaves_unmasked_envs_unchanged():
    w = world(4)
    w.reset()
    before = w.get_body_positions(zero_copy=False)
    mask = np.array([1, 0, 1, 0], np.uint8)
    for _ in range(20):
        w.step_subset(np.ones((4, w.action_dim), np.float32), mask)
    after = w.get_body_positions(zero_copy=False)
    assert not np.array_equal(before[0], after[0]) and not np.array_equal(before[2], after[2])
    np.testing.assert_array_equal(before[1], after[1])
    np.testing.assert_array_equal(before[3], after[3])


def test_masked_reset():
    n = 8
    w = world(n)
    w.reset()
    for _ in range(20):
        w.step(np.ones((n, w.action_dim), np.float32))
    before = w.get_body_positions(zero_copy=False)
    mask = np.zeros(n, np.uint8)
    mask[[0, 2, 4]] = 1
    w.reset(mask=mask)
    after = w.get_body_positions(zero_copy=False)
    for i in (0, 2, 4):
        assert not np.array_equal(before[i], after[i])
    for i in (1, 3, 5, 6, 7):
        np.testing.assert_array_equal(before[i], after[i])
    w.reset(mask=None)
    assert (w.get_contact_counts() == 0).all()


@pytest.mark.parametrize("value", [1e6, -1e6, 0.0])
def test_extreme_actions_stay_finite(value):
    w = world(1)
    w.reset()
    for _ in range(50 if value == 0 else 1):
        w.step(np.full((1, w.action_dim), value, np.float32))
    assert np.isfinite(w.get_observations()).all()


def test_nan_actions_and_dtype_coercion():
    w = world(1)
    w.reset()
    w.step(np.full((1, w.action_dim), np.nan, np.float32))
    assert w.get_observations() is not None
    w.step(np.zeros((1, w.action_dim), np.float64))
    assert w.get_observations().dtype == np.float32


def test_state_roundtrip():
    w = world(2)
    w.reset()
    a = np.full((2, w.action_dim), 0.5, np.float32)
    for _ in range(20):
        w.step(a)
    st = w.get_state()
    for _ in range(20):
        w.step(a)
    w.set_state(st)
    np.testing.assert_array_almost_equal(w.get_body_positions(zero_copy=False), st["body_positions"])


def test_gravity_and_timestep():
    w = world(1)
    w.reset()
    w.set_gravity((0.0, 0.0, 0.0))
    before = w.get_body_positions(zero_copy=False)
    for _ in range(50):
        w.step(np.zeros((1, w.action_dim), np.float32))
    after = w.get_body_positions(zero_copy=False)
    assert (np.abs(after[0, :, 2] - before[0, :, 2]) < 0.5).all()
    w2 = world(1)
    w2.set_timestep(0.001)
    assert w2.timestep == pytest.approx(0.001, rel=1e-5)
    w2.step(np.zeros((1, w2.action_dim), np.float32))
    assert np.isfinite(w2.get_observations()).all()
    with pytest.raises(RuntimeError):
        w2.set_timestep(0.0)


def test_accelerations_sensors_profiling():
    w = world(2, enable_profiling=True)
    w.reset()
    w.step(np.ones((2, w.action_dim), np.float32))
    acc = w.get_body_accelerations()
    assert acc.shape == (2, w.num_bodies, 4) and np.isfinite(acc).all()
    assert w.get_sensor_data().shape == (2, w.obs_dim)
    prof = w.get_profiling_data()
    assert prof["total_step_ms"] >= 0 and prof["num_active_constraints"] == 2 * 4
    w.reset_profiling()


@pytest.mark.parametrize("name", list(scenes.BY_NAME))
def test_every_scene_loads_and_steps(name):
    xml = scenes.BY_NAME[name]()
    kw = dict(max_contacts_per_env=256) if name == "collision_stress" else {}
    w = ZenoWorld(mjcf_string=xml, num_envs=2, **kw)
    w.reset()
    for _ in range(10):
        w.step(np.zeros((2, w.action_dim), np.float32))
    obs = w.get_observations()
    assert obs.shape == (2, w.obs_dim) and np.isfinite(obs).all()


def test_make_and_device_views():
    import torch
    env = zeno_b200.make("ant", num_envs=64, substeps=4)
    env.reset()
    w = env.world
    obs_t = torch.as_tensor(w.device_array("observations"), device="cuda")
    s = torch.cuda.Stream()
    w.set_stream(s.cuda_stream)
    acts = torch.rand((64, 8), device="cuda") * 2 - 1
    with torch.cuda.stream(s):
        w.step_async(acts)
    s.synchronize()
    np.testing.assert_array_equal(obs_t.cpu().numpy(), w.get_observations())


def test_output_host_copies_follow_the_device_buffers():
    """The host getters return pinned copies of the device outputs, refreshed by the first
    read after a step; rewards and dones are refreshed only when a step writes them (with
    the task on), so without the task a host write persists as in the reference, whose
    kernels never write them."""
    import torch
    w = ZenoWorld(mjcf_string=scenes.ant(), num_envs=256, substeps=4)
    w.reset()
    dev = {k: torch.as_tensor(w.device_array(k), device="cuda") for k in ("observations", "rewards", "dones")}
    rng = np.random.default_rng(3)
    o_zc = w.get_observations(zero_copy=True)
    for s in range(3):
        w.step(rng.uniform(-1, 1, (256, w.action_dim)).astype(np.float32))
        w.step(rng.uniform(-1, 1, (256, w.action_dim)).astype(np.float32))  # two steps, one read
        obs = w.get_observations()
        np.testing.assert_array_equal(obs, dev["observations"].cpu().numpy())
        np.testing.assert_array_equal(o_zc, obs)  # the same host buffer
        np.testing.assert_array_equal(w.get_sensor_data(), obs)
    rew = w._view(zeno_b200._ffi._lib.zeno_world_get_rewards(w.handle), (256,))
    rew[:] = 7.0
    w.step(np.zeros((256, w.action_dim), np.float32))
    assert (w.get_rewards() == 7.0).all()
    w.set_task(auto_reset=False, z_min=0.2, z_max=10.0)
    w.step(np.zeros((256, w.action_dim), np.float32))
    np.testing.assert_array_equal(w.get_rewards(), dev["rewards"].cpu().numpy())
    np.testing.assert_array_equal(w.get_dones(), dev["dones"].cpu().numpy())
    assert not (w.get_rewards() == 7.0).any()
