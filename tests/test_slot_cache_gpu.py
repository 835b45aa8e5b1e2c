"""The compressed-state kernel's slot cache: its own copy of every environment's contact
list, used in place of the contact records until the caller is handed the contacts
buffer (zeno_world_get_contacts), after which the records are read again every step.

These tests compare every ABI buffer except the contact records step by step (reading
them through zeno_world_get_contacts would end the cache's use), and the records at the
end, over the paths that change what the cache holds: long runs with device resets,
subset steps, resets from the host, narrow-phase and kernel switches."""
import numpy as np
import pytest

from parity import FIELDS, actions, diff_report, make_pair, product_state

pytestmark = pytest.mark.gpu

NO_CONTACTS = [f for f in FIELDS if f != "contacts"]


def state_without_records(w):
    """product_state minus the contact records (the counters are a separate buffer)."""
    return {
        "positions": w.get_body_positions(zero_copy=False),
        "quaternions": w.get_body_quaternions(zero_copy=False),
        "velocities": w.get_body_velocities(zero_copy=False),
        "angular_velocities": w.get_body_angular_velocities(zero_copy=False),
        "accelerations": w.get_body_accelerations(zero_copy=False),
        "joint_positions": w.get_joint_positions(zero_copy=False),
        "joint_velocities": w.get_joint_velocities(zero_copy=False),
        "joint_torques": w.get_joint_forces(zero_copy=False),
        "observations": w.get_observations(zero_copy=False),
        "rewards": w.get_rewards(),
        "dones": w.get_dones(),
        "contact_counts": w.get_contact_counts(),
    }


def check(w, o, s, fields=NO_CONTACTS):
    bad = diff_report(state_without_records(w) if "contacts" not in fields else product_state(w), o.state(), fields)
    assert not bad, f"step {s}: {bad}"


@pytest.mark.parametrize("name", ["ant", "humanoid"])
def test_long_run_with_device_resets(name):
    E, N = 64, 150
    w, o, c = make_pair(name, E)
    for x in (w, o):
        x.set_task(body=1, z_min=0.2 if name == "ant" else 1.0, z_max=1.0 if name == "ant" else np.inf,
                   auto_reset=True, noise=0.1, seed=3)
    acts = actions(np.random.default_rng(4), N, E, w.action_dim, c["act"])
    for s in range(N):
        w.step(acts[s])
        o.step(acts[s])
        if s % 25 == 0:
            check(w, o, s)
    assert int(w.get_dones().sum()) >= 0
    check(w, o, N, FIELDS)  # the records too (from here on they are read every step)
    for s in range(5):
        w.step(acts[s])
        o.step(acts[s])
        check(w, o, N + s, FIELDS)


def test_subset_steps_and_host_resets():
    E = 16
    w, o, c = make_pair("ant", E)
    rng = np.random.default_rng(12)
    acts = actions(rng, 40, E, w.action_dim, c["act"])
    for s in range(40):
        if s % 5 == 2:
            mask = (rng.random(E) < 0.5).astype(np.uint8)
            w.step_subset(acts[s], mask)
            o.step_subset(acts[s], mask)
        else:
            w.step(acts[s])
            o.step(acts[s])
        if s == 11:
            m = np.zeros(E, np.uint8)
            m[[1, 4, 9]] = 1
            w.reset(m)
            o.reset(m)
        if s == 23:
            st = state_without_records(w)
            w.reset_to_state(st["positions"], st["quaternions"], None, None, None)
            o.reset_to_state(st["positions"], st["quaternions"], None, None, None)
        check(w, o, s)
    check(w, o, 40, FIELDS)


def test_kernel_and_narrow_phase_switches():
    """Steps on the general kernel and a narrow-phase change leave the cache stale; the
    fast kernel must then read the records."""
    E = 16
    w, o, c = make_pair("ant", E)
    acts = actions(np.random.default_rng(8), 30, E, w.action_dim, c["act"])
    fast = w.get_launch()
    for s in range(30):
        if s == 8:
            w.set_launch(8, 4)
        if s == 12:
            w.set_launch(*fast)
        if s == 18:
            w.set_narrow_phase(1)
            o.set_narrow_phase(1)
        if s == 24:
            w.set_narrow_phase(0)
            o.set_narrow_phase(0)
        w.step(acts[s])
        o.step(acts[s])
        check(w, o, s)
    check(w, o, 30, FIELDS)


def test_host_writes_after_exposure_are_read():
    """Once the contacts buffer was handed out, a host write to a record counts: an
    impulse written into a live slot warm-starts the next step as in the oracle."""
    E = 4
    w, o, c = make_pair("ant", E)
    acts = actions(np.random.default_rng(2), 6, E, w.action_dim, c["act"])
    for s in range(3):
        w.step(acts[s])
        o.step(acts[s])
    rec = w.get_contacts(zero_copy=True)
    orec = o.raw("contacts", rec.dtype).reshape(E, -1)
    for arr in (rec, orec):
        arr["impulses"][:, :8, 0] = 0.25
    for s in range(3, 6):
        w.step(acts[s])
        o.step(acts[s])
        check(w, o, s, FIELDS)
