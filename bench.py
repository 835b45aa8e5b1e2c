"""Benchmark: Ant env-steps/s (16384 envs per GPU) and the step's HBM-roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE Ant config): the reference Ant model, dt 0.01 s, 4 substeps, 4 solver
iterations, 64 contact slots per env, 16384 envs per GPU, actions U(-1, 1) drawn from a
seeded generator, done = torso z outside [0.2, 1.0] with device-side masked reset and
U(-0.1, 0.1) pose noise.  Synthetic inputs only; no datasets.

One "step" is one World.step over all envs of a GPU (one fused kernel launch, plus the
hand-over launch that steps environments the fast kernel could not represent).  `value`
is the whole-job throughput with actions already resident in HBM, timed with CUDA
events on the launching stream around each step; L2 is flushed (a 256 MiB write)
between timed steps, outside the events.  `e2e` is the same metric through the
reference-facing API with host buffers: per step, actions are copied from pinned host
memory by zeno_world_step and observations, rewards and dones are read back into host
arrays.  Multi-GPU runs are one process per GPU (torchrun); environments are sharded with
no collective on the step path (weak scaling); timings are the max over ranks.

Every workload starts from the model pose with joint-coordinate noise (BASELINE: Ant
U(-0.1, 0.1), Humanoid U(-0.01, 0.01), Pendulum hinge U(-0.1, 0.1), Cartpole qpos and qvel
U(-0.01, 0.01)), applied by zeno_b200.initial_state and zeno_world_reset_to_state.

--impl reference times the reference algorithm on the host CPU cores: the reference
implementation cannot run here (its step exists only as Metal shaders), so the CPU
restatement in oracle/ is timed with all host threads, each step one World.step over a
sample of the workload's environments sized so the timed steps take at least 6 s, with
the same settings, initial state, task and `config` as the GPU arm.  That arm loads no
product library.

Other workloads (not the headline line; same JSON contract): --scene pendulum (BASELINE
config 1: 1024 envs, dt 0.01 s, 4 substeps, no contacts), --scene cartpole (config 2:
4096 envs, dt 0.01 s, 1 substep), --scene humanoid (the
reference Humanoid, dt 0.015 s, 4 substeps, actions U(-0.4, 0.4), done = torso z < 1.0 with
U(-0.01, 0.01) reset noise) or --scene collision_stress (the seeded 64-body drop scene,
4096 envs per GPU, dt 0.005 s, 8 substeps, 256 contact slots, no actuators); --narrow 0/1/2
selects the narrow phase and --semantics corrected the corrected-semantics mode;
--scene sphere_pile (600 free spheres, 1024 envs per GPU, 1024 contact slots: past the
reference's 512-geom switch to its spatial hash) with --broad 1 (all candidate pairs) or
--broad 2 (hashed grid; the default above 512 geoms) times the broad phases.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ENVS_PER_GPU = 16384
ACTION_RING = 64   # distinct pre-generated action batches, resident in HBM, cycled over the steps
E2E_STEPS = 200    # steps of the end-to-end leg
CPU_SAMPLE_ENVS = 2048  # cpu_baseline: envs stepped by the CPU oracle ...
CPU_SAMPLE_S = 10.0     # ... for about this many seconds
REF_TARGET_S = 6.0      # --impl reference: the timed steps take at least this long
SUBSTEPS = 4
ITERATIONS = 4
MAX_CONTACTS = 64
METRIC = "env-steps/sec (whole box, Ant 16384 envs/GPU)"
UNIT = "env-steps/s"


def scene_config(name: str) -> dict:
    """Per-workload settings: envs per GPU, timestep, substeps, solver iterations, contact
    slots, action scale, initial joint-coordinate noise (qpos, qvel) or None, and the task
    (done rule and reset noise) or None."""
    from zeno_b200 import scenes  # pure Python: does not load libzeno.so
    inf = float("inf")
    return {
        "ant": dict(xml=scenes.ant, envs=ENVS_PER_GPU, timestep=0.01, substeps=SUBSTEPS, iters=ITERATIONS,
                    M=MAX_CONTACTS, act=1.0, init=(0.1, 0.0), task=dict(body=1, z_min=0.2, z_max=1.0, noise=0.1),
                    task_text="done: torso z not in [0.2, 1.0], device auto-reset, U(-0.1,0.1) noise"),
        "humanoid": dict(xml=scenes.humanoid, envs=ENVS_PER_GPU, timestep=0.015, substeps=4, iters=4, M=64,
                         act=0.4, init=(0.01, 0.0), task=dict(body=1, z_min=1.0, z_max=inf, noise=0.01),
                         task_text="done: torso z < 1.0, device auto-reset, U(-0.01,0.01) noise"),
        "pendulum": dict(xml=scenes.pendulum, envs=1024, timestep=0.01, substeps=4, iters=4, M=64, act=1.0,
                         init=(0.1, 0.0), task=None, task_text="none (no contacts; hinge angle U(-0.1,0.1) at start)"),
        "cartpole": dict(xml=scenes.cartpole, envs=4096, timestep=0.01, substeps=1, iters=4, M=64, act=1.0,
                         init=(0.01, 0.01), task=None, task_text="none (qpos, qvel U(-0.01,0.01) at start)"),
        "collision_stress": dict(xml=lambda: scenes.collision_stress(0), envs=4096, timestep=0.005, substeps=8,
                                 iters=4, M=256, act=0.0, init=None, task=None,
                                 task_text="none (free fall, no actuators)"),
        "sphere_pile": dict(xml=lambda: scenes.sphere_pile(0), envs=1024, timestep=0.005, substeps=4, iters=4,
                            M=1024, act=0.0, init=None, task=None, task_text="none (600 free spheres, no actuators)"),
    }[name]


def initial_state(tables, pos0, quat0, sc, E, rank):
    """Per-environment initial body state: the model pose with the workload's joint-coordinate
    noise (zeno_b200.initial_state), seeded by rank so shards differ; None without noise."""
    if not sc["init"]:
        return None
    from zeno_b200.initial_state import joint_noise_state
    qpos, qvel = sc["init"]
    return joint_noise_state(tables["bodies"], tables["joints"], pos0, quat0, E,
                             np.random.default_rng(1000 + rank), qpos, qvel)


def bench_config(args, sc, E, world_size):
    """The workload's `config` object, identical in both arms."""
    narrow = args.narrow if args.narrow is not None else (2 if args.semantics == "corrected" else 0)
    return {"workload": workload_name(args), "envs_per_gpu": E, "substeps": sc["substeps"],
            "contact_iterations": sc["iters"], "max_contacts_per_env": sc["M"], "timestep": sc["timestep"],
            "narrow_phase": narrow, "semantics": args.semantics,
            "broad_phase": args.broad if args.broad is not None else 0,
            "initial_noise": (f"joint coordinates U(-{sc['init'][0]},{sc['init'][0]})"
                              + (f", rates U(-{sc['init'][1]},{sc['init'][1]})" if sc["init"][1] else "")
                              ) if sc["init"] else "none",
            "task": sc["task_text"],
            "actions": f"U(-{sc['act']},{sc['act']}) per env per step" if sc["act"] else "none",
            "l2": "flushed (256 MiB write) between timed steps",
            "parallelism": f"env-sharded x{world_size}, no collective on the step path"}


def algorithmic_bytes_per_env_step(B, J, A, obs, K, S):
    """Bytes one env-step must move to and from HBM (per-unit figure of the roofline):
    actions R, pos/quat/vel/angvel R+W, accel W, joint pos/vel/torque W, observations W,
    reward+done W, contact count and previous count R+W, S contact slots R+W, and the
    constraint multipliers (lambda, lambda_prev) R+W."""
    return 4 * A + 128 * B + 16 * B + 12 * J + 4 * obs + 5 + 16 + 128 * S + 16 * K


def shard_env_offset(rank: int, envs_per_gpu: int) -> int:
    """Global index of a rank's first env.  Envs are sharded in contiguous blocks; the
    offset keys the reset-noise generator, so an env's trajectory does not depend on how
    many GPUs share the job."""
    return rank * envs_per_gpu


def reduce_max(value: float, dist, device) -> float:
    """Max over ranks (the timing rule for multi-GPU runs)."""
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            t0 = time.perf_counter()  # the timed region starts once the sampler is reporting
            while not self.lines and time.perf_counter() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.lines.clear()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


TRAFFIC_FILE = ROOT / "profiles" / "step_traffic.json"


def dram_bytes_per_launch(kernel: str, scene: str, envs: int):
    """DRAM bytes (read + write) per launch of `kernel` on `scene`, from the ncu capture
    recorded in profiles/step_traffic.json (written by `bench.py --record-traffic`), scaled
    to `envs` environments (the traffic is per environment); None when not recorded."""
    if not TRAFFIC_FILE.exists():
        return None
    for r in json.loads(TRAFFIC_FILE.read_text()).get("captures", []):
        if r["kernel"] == kernel and r["scene"] == scene:
            return float(r["dram_bytes_per_launch"]) * envs / int(r["envs"])
    return None


def record_traffic(csv_path: str, scene: str, envs: int, command: str) -> None:
    """Reads an ncu raw-page CSV (`ncu -i <rep> --page raw --csv`) and records, per step
    kernel, dram__bytes_read.sum + dram__bytes_write.sum averaged over its captured
    launches into profiles/step_traffic.json (replacing the entry of the same kernel and
    scene)."""
    import csv
    rows = list(csv.reader(open(csv_path)))
    head = rows[0]
    idx = {k: head.index(k) for k in ("Kernel Name", "dram__bytes_read.sum", "dram__bytes_write.sum")}
    units = rows[1] if len(rows) > 1 and not rows[1][idx["Kernel Name"]] else None
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9}
    import re
    per = {}
    for r in rows[2 if units else 1:]:
        km = re.search(r"\b(fast_step_kernel|step_kernel)<(\d+)", r[idx["Kernel Name"]])
        if not km:
            continue
        k = f"zb::{km.group(1)}<{km.group(2)}>"  # the name bench.py reports (lanes only)
        tot = 0.0
        for m in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            u = units[idx[m]] if units else "byte"
            tot += float(r[idx[m]].replace(",", "")) * scale.get(u, 1)
        per.setdefault(k, []).append(tot)
    data = json.loads(TRAFFIC_FILE.read_text()) if TRAFFIC_FILE.exists() else {"captures": []}
    for k, v in per.items():
        data["captures"] = [c for c in data["captures"] if not (c["kernel"] == k and c["scene"] == scene)]
        data["captures"].append({"kernel": k, "scene": scene, "envs": envs, "launches": len(v),
                                 "dram_bytes_per_launch": sum(v) / len(v), "command": command})
    TRAFFIC_FILE.write_text(json.dumps(data, indent=1) + "\n")


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def oracle_world(xml, sc, envs, narrow=None, semantics="reference", rank=0):
    """The CPU oracle set up like the GPU arm's world: same settings, initial state and task."""
    from oracle.zeno_oracle import OracleWorld
    o = OracleWorld(xml, num_envs=envs, timestep=sc["timestep"], substeps=sc["substeps"],
                    contact_iterations=sc["iters"], max_contacts_per_env=sc["M"], semantics=semantics)
    if narrow is not None:
        o.set_narrow_phase(narrow)
    st = o.state()
    init = initial_state({"bodies": o.model_table("bodies"), "joints": o.model_table("joints")},
                         st["positions"][0], st["quaternions"][0], sc, envs, rank)
    if init is not None:
        o.reset_to_state(init["positions"], init["quaternions"], init["velocities"], init["angular_velocities"])
    if sc["task"]:
        o.set_task(auto_reset=True, seed=1, **sc["task"])
    return o


def time_oracle(o, sc, threads, warmup=1, steps=0, target_s=0.0):
    """Steps the oracle world `o` (actions U(-act, act), a ring of distinct batches): `warmup`
    untimed steps, then `steps` timed steps, repeated until at least `target_s` seconds have
    passed.  Returns (env-steps/s, seconds, steps timed)."""
    rng = np.random.default_rng(0)
    A = max(o.num_actuators, 1)
    ring = (sc["act"] * rng.uniform(-1, 1, size=(min(max(steps, 10), ACTION_RING), o.num_envs, A))).astype(np.float32)
    for k in range(warmup):
        o.run(ring[k % len(ring)][None], threads=threads)
    batch = max(steps, 10)
    done = 0
    t0 = time.perf_counter()
    while True:
        for k in range(0, batch, len(ring)):
            n = min(len(ring), batch - k)
            o.run(ring[:n], threads=threads)
        done += batch
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    return done * o.num_envs / dt, dt, done


def cpu_baseline(xml, sc, sample_envs, threads, target_s, narrow=None, semantics="reference"):
    """The cpu_baseline leg: the CPU oracle on a bounded sample of the workload's envs for
    about target_s seconds.  Returns (env-steps/s, seconds, steps run)."""
    o = oracle_world(xml, sc, sample_envs, narrow, semantics)
    return time_oracle(o, sc, threads, warmup=1, steps=10, target_s=target_s)


def metric_name(args, E):
    if args.scene == "ant" and args.narrow is None and args.semantics == "reference" and args.broad is None:
        return METRIC
    return f"env-steps/sec (whole box, {args.scene} {E} envs/GPU)"


def workload_name(args):
    w = args.scene
    if args.broad is not None:
        w += f", broad phase {args.broad}"
    if args.narrow is not None:
        w += f", narrow phase {args.narrow}"
    if args.semantics != "reference":
        w += f", {args.semantics} semantics"
    return w


def run_reference(args, rank, world_size):
    """The reference arm: the reference's step algorithm on the host cores.  The reference
    step exists only as Metal shaders and its Zig host cannot be built here, so the CPU
    restatement in oracle/ stands in for it (the same arithmetic and step order the GPU is
    checked against bit for bit), on all host threads.  One step = one World.step over a
    sample of the workload's environments, sized so the K timed steps take at least
    REF_TARGET_S seconds (all of them repeated when even the full workload is faster).
    This arm loads no product library: scenes and initial_state are pure Python."""
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    sc = scene_config(args.scene)
    E = args.envs or sc["envs"]
    xml = sc["xml"]()
    narrow = args.narrow
    probe = oracle_world(xml, sc, min(256, E), narrow, args.semantics)
    rate, _, _ = time_oracle(probe, sc, threads, warmup=2, steps=10, target_s=0.5)
    del probe
    sample = int(min(E, max(64, np.ceil(REF_TARGET_S * rate / max(args.steps, 1)))))
    o = oracle_world(xml, sc, sample, narrow, args.semantics)
    val, dt, done = time_oracle(o, sc, threads, warmup=args.warmup, steps=args.steps, target_s=REF_TARGET_S)
    line = {
        "impl": "reference", "metric": metric_name(args, E), "value": val, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / done, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(args, sc, E, world_size),
        "sample_envs_per_step": sample, "timed_steps": done,
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} of {E} {args.scene} envs per step x {done} steps on {threads} threads "
                                   f"({dt:.1f} s); the reference step exists only as Metal shaders, so the CPU "
                                   "restatement in oracle/ stands in for it"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_e2e(w, pinned, acts, args, E, A, dist, barrier, world_size, torch):
    """Same metric through the reference-facing API: zeno_world_step with host actions
    (pinned), then observations, rewards and dones read into host arrays (observations as
    the reference API's zero_copy view of the host copy the step just filled by DMA, so
    the wrapper does not copy 1.9 MB a second time; rewards and dones as copies)."""
    pinned.copy_(acts.cpu())
    host_acts = pinned.numpy()
    ring = host_acts.shape[0]
    steps = min(args.steps, E2E_STEPS)
    w.set_stream(0)  # the public API runs on the world's own stream
    for s in range(2):
        w.step(host_acts[s])
        w.get_observations(zero_copy=True), w.get_rewards(), w.get_dones()
    barrier()
    e0 = time.perf_counter()
    for s in range(steps):
        w.step(host_acts[s % ring])
        obs = w.get_observations(zero_copy=True)
        rew = w.get_rewards()
        don = w.get_dones()
    e_local = time.perf_counter() - e0
    e2e_value = world_size * E * steps / reduce_max(e_local, dist, "cuda")
    h2d = E * A * 4
    d2h = obs.nbytes + rew.nbytes + don.nbytes
    return e2e_value, h2d, int(d2h)


def run_gather(w, dist, barrier, torch, reps=20):
    """All-gather of every rank's observations, rewards and dones (zeno_b200.gather, NCCL
    over NVLink / NVSwitch), timed with events on the gather's stream, max over ranks."""
    from zeno_b200.gather import OutputGather
    g = OutputGather.for_world(w)
    for _ in range(3):
        g.all_gather()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(g.stream)
    for _ in range(reps):
        g.all_gather()
    e1.record(g.stream)
    e1.synchronize()
    ms = reduce_max(e0.elapsed_time(e1) / reps, dist, "cuda")
    per_rank = sum(t.numel() * t.element_size() for t in g.inputs)
    total = sum(t.numel() * t.element_size() for t in g.outputs)
    return {"op": "all_gather of observations, rewards, dones onto every rank (NCCL), outside the timed steps",
            "ms": ms, "bytes_per_rank": per_rank, "bytes_gathered": total,
            "algbw_GBps": total / (ms / 1000.0) / 1e9}


def run_ours(args, rank, world_size, local_rank):
    import torch

    import zeno_b200
    from zeno_b200 import scenes

    torch.cuda.set_device(local_rank)
    dist = None
    if world_size > 1:
        import torch.distributed as dist_
        from datetime import timedelta
        dist_.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
        dist = dist_

    sc = scene_config(args.scene)
    E = args.envs or sc["envs"]
    xml = sc["xml"]()
    w = zeno_b200.ZenoWorld(mjcf_string=xml, num_envs=E, timestep=sc["timestep"], substeps=sc["substeps"],
                            contact_iterations=sc["iters"], max_contacts_per_env=sc["M"], semantics=args.semantics)
    if args.narrow is not None:
        w.set_narrow_phase(args.narrow)
    if args.broad is not None:
        w.set_broad_phase(args.broad)
    if args.launch:
        lanes, epb = (int(x) for x in args.launch.split(","))
        w.set_launch(lanes, epb)
    config = bench_config(args, sc, E, world_size)
    if (w.get_narrow_phase(), w.get_broad_phase()) != (config["narrow_phase"], config["broad_phase"]):
        raise RuntimeError("world settings differ from the reported config")
    init = initial_state({"bodies": w.model_table("bodies"), "joints": w.model_table("joints")},
                         w.get_body_positions(zero_copy=False)[0], w.get_body_quaternions(zero_copy=False)[0],
                         sc, E, rank)
    if init is not None:
        w.reset_to_state(init["positions"], init["quaternions"], init["velocities"], init["angular_velocities"])
    if sc["task"]:
        w.set_task(auto_reset=True, seed=1, env_offset=shard_env_offset(rank, E), **sc["task"])
    # a dedicated stream: the world launches on it and the timing events record on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    w.set_stream(stream.cuda_stream)
    A = w.action_dim

    # inputs resident in HBM before timing: one action batch per step
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    total = args.warmup + args.steps
    ring = min(total, ACTION_RING)  # distinct action batches, cycled
    acts = (torch.rand((ring, E, A), device="cuda", generator=gen, dtype=torch.float32) * 2 - 1) * sc["act"]
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MiB > 126 MB L2

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for s in range(args.warmup):
        w.step_async(acts[s % ring])
    barrier()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        barrier()
        wall0 = time.perf_counter()
        for s in range(args.steps):
            flush.zero_()
            starts[s].record(stream)
            w.step_async(acts[(args.warmup + s) % ring])
            ends[s].record(stream)
        barrier()
        wall = time.perf_counter() - wall0
    step_ms = [starts[s].elapsed_time(ends[s]) for s in range(args.steps)]
    t_local = sum(step_ms) / 1000.0
    t_max = reduce_max(t_local, dist, "cuda")
    value = world_size * E * args.steps / t_max
    dones_seen = int(w.get_dones().sum())

    # ---- end to end through the reference-facing API, host buffers ----
    e2e_value, h2d, d2h = None, E * A * 4, 0
    if args.no_e2e:
        pinned = None
    else:
        pinned = torch.empty((ring, E, A), dtype=torch.float32, pin_memory=True)
    if pinned is not None:
        e2e_value, h2d, d2h = run_e2e(w, pinned, acts, args, E, A, dist, barrier, world_size, torch)

    # ---- optional output gather (NCCL), after and outside the timed steps ----
    gather = run_gather(w, dist, barrier, torch) if args.gather and dist else None

    if rank == 0:
        st = w.get_info()
        counts = w.get_contact_counts()
        obs_dim, B, J = w.obs_dim, w.num_bodies, w.num_joints
        try:
            K = len(w.model_table("constraints")) // 96
        except KeyError:  # no constraints (free bodies only)
            K = 0
        live_slots = float(np.minimum(counts, sc["M"]).mean())  # S: the slots the step reads and writes
        bpe = algorithmic_bytes_per_env_step(B, J, A, obs_dim, K, live_slots)
        mean_ms = statistics.mean(step_ms)
        achieved = bpe * E / (mean_ms / 1000.0) / 1e9
        peak, peak_kind = measured_peaks()
        lanes, epb = w.get_launch()
        kernel = f"zb::fast_step_kernel<{lanes}>" if lanes in (1, 2, 4) else f"zb::step_kernel<{lanes}>"
        traffic = dram_bytes_per_launch(kernel, args.scene, E)
        cpu_envs = min(CPU_SAMPLE_ENVS, E)
        cpu_val, cpu_dt, cpu_steps = (cpu_baseline(xml, sc, cpu_envs, os.cpu_count() or 1, CPU_SAMPLE_S,
                                                   narrow=args.narrow, semantics=args.semantics)
                                      if not args.no_cpu else (None, 0, 0))
        clocks = clk.summary()
        line = {
            "metric": metric_name(args, E), "value": value, "unit": UNIT, "n_gpus": world_size, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max * 1000.0 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config,
            "launch": {"lanes_per_env": lanes, "envs_per_block": epb},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "bytes_per_env_step": bpe, "kernel": kernel,
                         "mean_launch_ms": mean_ms},
            "cpu_baseline": {"value": cpu_val, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": f"{cpu_envs} {args.scene} envs x {cpu_steps} steps, oracle on "
                                       f"{os.cpu_count()} threads ({cpu_dt:.1f} s)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": int(d2h)},
            # per step: the step kernel, plus (environment-per-lane kernel) the hand-over
            # launch of the general kernel, which exits at once when nothing was handed over
            "gpu_launches": args.steps * (2 if lanes in (1, 2, 4) else 1),
            "clocks": clocks,
            "wall_s_timed_region": wall,
            "dones_in_last_step": dones_seen,
            "mean_contact_count": float(counts.mean()),
        }
        if gather:
            line["gather"] = gather
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_stage_profile(args):
    """Per-stage device cycles of the step (a profiling world: the instrumented kernel
    instantiation, zeno_world_get_stage_cycles), averaged over the timed steps; one JSON
    line.  Not a throughput measurement: the instrumented kernel is slower."""
    import torch

    import zeno_b200
    torch.cuda.set_device(0)
    sc = scene_config(args.scene)
    E = args.envs or sc["envs"]
    w = zeno_b200.ZenoWorld(mjcf_string=sc["xml"](), num_envs=E, timestep=sc["timestep"], substeps=sc["substeps"],
                            contact_iterations=sc["iters"], max_contacts_per_env=sc["M"], semantics=args.semantics,
                            enable_profiling=True)
    if args.narrow is not None:
        w.set_narrow_phase(args.narrow)
    if args.launch:
        w.set_launch(*(int(x) for x in args.launch.split(",")))
    init = initial_state({"bodies": w.model_table("bodies"), "joints": w.model_table("joints")},
                         w.get_body_positions(zero_copy=False)[0], w.get_body_quaternions(zero_copy=False)[0],
                         sc, E, 0)
    if init is not None:
        w.reset_to_state(init["positions"], init["quaternions"], init["velocities"], init["angular_velocities"])
    if sc["task"]:
        w.set_task(auto_reset=True, seed=1, **sc["task"])
    rng = np.random.default_rng(0)
    acc = {}
    for s in range(args.warmup + args.steps):
        a = (sc["act"] * rng.uniform(-1, 1, size=(E, max(w.action_dim, 1)))).astype(np.float32)
        w.step(a)
        if s < args.warmup:
            continue
        prof = w.get_stage_profile()
        if not prof:
            raise RuntimeError("no stage profile returned")
        for k, v in prof.items():
            acc[k] = acc.get(k, 0.0) + v / args.steps
    lanes, epb = w.get_launch()
    print(json.dumps({"stage_profile": args.scene, "envs": E, "steps": args.steps, "launch": [lanes, epb],
                      "cycles_per_block_step": {k: round(v) for k, v in acc.items()
                                                if k != "ns_per_cycle" and not k.startswith("max_")},
                      "max_over_blocks": {k[4:]: round(v) for k, v in acc.items() if k.startswith("max_")},
                      "ns_per_cycle": acc.get("ns_per_cycle"), "profiling_data": w.get_profiling_data()}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) leg")
    ap.add_argument("--envs", type=int, default=0, help="environments per GPU (0: the workload's)")
    ap.add_argument("--scene", choices=["ant", "humanoid", "pendulum", "cartpole", "collision_stress", "sphere_pile"],
                    default="ant")
    ap.add_argument("--broad", type=int, choices=[0, 1, 2], default=None, help="broad phase (default: the world's)")
    ap.add_argument("--narrow", type=int, choices=[0, 1, 2], default=None, help="narrow phase (default: the world's)")
    ap.add_argument("--semantics", choices=["reference", "corrected"], default="reference")
    ap.add_argument("--gather", action="store_true",
                    help="with N > 1: also time the optional NCCL all-gather of the step outputs (not in value)")
    ap.add_argument("--launch", default="", help="launch shape 'lanes,envs_per_block' (default: the world's choice)")
    ap.add_argument("--stage-profile", action="store_true",
                    help="print per-stage device cycles of the step (instrumented kernel; no throughput line)")
    ap.add_argument("--record-traffic", nargs=4, metavar=("CSV", "SCENE", "ENVS", "COMMAND"),
                    help="record DRAM traffic per launch from an ncu raw CSV into profiles/step_traffic.json")
    args = ap.parse_args()
    if args.record_traffic:
        csv_path, scene, envs, command = args.record_traffic
        record_traffic(csv_path, scene, int(envs), command)
        return 0
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world_size)
    if args.stage_profile:
        return run_stage_profile(args)
    return run_ours(args, rank, world_size, local_rank)


if __name__ == "__main__":
    sys.exit(main())
