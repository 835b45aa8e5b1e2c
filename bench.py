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

--impl reference times the reference algorithm on the host CPU cores: the reference
implementation cannot run here (its step exists only as Metal shaders), so the CPU
restatement in oracle/ is timed with all host threads on a bounded sample of envs.

Other workloads (not the headline line; same JSON contract): --scene humanoid (the
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
SUBSTEPS = 4
ITERATIONS = 4
MAX_CONTACTS = 64
METRIC = "env-steps/sec (whole box, Ant 16384 envs/GPU)"
UNIT = "env-steps/s"


def scene_config(name: str) -> dict:
    """Per-workload settings: envs per GPU, timestep (0: the MJCF's), substeps, solver
    iterations, contact slots, action scale, the task (done rule and reset noise) or None."""
    from zeno_b200 import scenes
    inf = float("inf")
    return {
        "ant": dict(xml=scenes.ant, envs=ENVS_PER_GPU, timestep=0.0, substeps=SUBSTEPS, iters=ITERATIONS,
                    M=MAX_CONTACTS, act=1.0, task=dict(body=1, z_min=0.2, z_max=1.0, noise=0.1),
                    task_text="done: torso z not in [0.2, 1.0], device auto-reset, U(-0.1,0.1) noise"),
        "humanoid": dict(xml=scenes.humanoid, envs=ENVS_PER_GPU, timestep=0.015, substeps=4, iters=4, M=64,
                         act=0.4, task=dict(body=1, z_min=1.0, z_max=inf, noise=0.01),
                         task_text="done: torso z < 1.0, device auto-reset, U(-0.01,0.01) noise"),
        "collision_stress": dict(xml=lambda: scenes.collision_stress(0), envs=4096, timestep=0.005, substeps=8,
                                 iters=4, M=256, act=0.0, task=None, task_text="none (free fall, no actuators)"),
        "sphere_pile": dict(xml=lambda: scenes.sphere_pile(0), envs=1024, timestep=0.005, substeps=4, iters=4,
                            M=1024, act=0.0, task=None, task_text="none (600 free spheres, no actuators)"),
    }[name]


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


def dram_bytes_per_launch(kernel: str, envs: int):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu summary
    (profiles/step_traffic.md: a row `| kernel | envs | dram_bytes_per_launch |`), scaled to
    `envs` environments (traffic is per environment), or None."""
    import re
    for f in sorted((ROOT / "profiles").glob("*_traffic.md")):
        for line in f.read_text().splitlines():
            m = re.match(r"\|\s*(\S+)\s*\|\s*(\d+)\s*\|\s*([\d.]+)\s*\|", line)
            if m and m.group(1) == kernel:
                return float(m.group(3)) * envs / int(m.group(2))
    return None


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def cpu_baseline(xml, steps, sample_envs, threads, target_s=None, sc=None, narrow=None, semantics="reference"):
    """The CPU oracle (reference algorithm restated) on a bounded sample of envs: `steps`
    steps, or (target_s set) as many 10-step batches as fill about target_s seconds.
    Returns (env-steps/s, seconds, steps run)."""
    from oracle.zeno_oracle import OracleWorld
    sc = sc or scene_config("ant")
    o = OracleWorld(xml, num_envs=sample_envs, timestep=sc["timestep"], substeps=sc["substeps"],
                    contact_iterations=sc["iters"], max_contacts_per_env=sc["M"], semantics=semantics)
    if narrow is not None:
        o.set_narrow_phase(narrow)
    if sc["task"]:
        o.set_task(auto_reset=True, seed=1, **sc["task"])
    rng = np.random.default_rng(0)
    batch = 10 if target_s else steps
    acts = (sc["act"] * rng.uniform(-1, 1, size=(batch, sample_envs, o.num_actuators))).astype(np.float32)
    o.run(acts[:1], threads=threads)  # warm-up
    done = 0
    t0 = time.perf_counter()
    while True:
        o.run(acts, threads=threads)
        done += batch
        dt = time.perf_counter() - t0
        if not target_s or dt >= target_s:
            break
    return done * sample_envs / dt, dt, done


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


def run_reference(args, rank):
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    sc = scene_config(args.scene)
    sample = min(2048, sc["envs"])
    xml = sc["xml"]()
    val, dt, _ = cpu_baseline(xml, args.warmup + args.steps, sample, threads, sc=sc, narrow=args.narrow,
                              semantics=args.semantics)
    line = {
        "impl": "reference", "metric": metric_name(args, sc["envs"]), "value": val, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * sample / val, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args), "envs_per_gpu": sc["envs"], "substeps": sc["substeps"],
                   "contact_iterations": sc["iters"], "max_contacts_per_env": sc["M"],
                   "sample_envs_per_step": sample},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} {args.scene} envs x {args.warmup + args.steps} steps on {threads} threads "
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
        bpe = algorithmic_bytes_per_env_step(B, J, A, obs_dim, K, sc["M"])
        mean_ms = statistics.mean(step_ms)
        achieved = bpe * E / (mean_ms / 1000.0) / 1e9
        peak, peak_kind = measured_peaks()
        lanes, epb = w.get_launch()
        kernel = f"zb::fast_step_kernel<{lanes}>" if lanes in (1, 2, 4) else f"zb::step_kernel<{lanes}>"
        traffic = dram_bytes_per_launch(kernel, E)
        cpu_envs = min(CPU_SAMPLE_ENVS, E)
        cpu_val, cpu_dt, cpu_steps = (cpu_baseline(xml, 0, cpu_envs, os.cpu_count() or 1, CPU_SAMPLE_S, sc=sc,
                                                   narrow=args.narrow, semantics=args.semantics)
                                      if not args.no_cpu else (None, 0, 0))
        clocks = clk.summary()
        line = {
            "metric": metric_name(args, E), "value": value, "unit": UNIT, "n_gpus": world_size, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max * 1000.0 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload_name(args), "envs_per_gpu": E, "substeps": sc["substeps"],
                       "contact_iterations": sc["iters"], "max_contacts_per_env": sc["M"], "timestep": st["timestep"],
                       "narrow_phase": w.get_narrow_phase(), "semantics": args.semantics,
                       "broad_phase": w.get_broad_phase(),
                       "task": sc["task_text"],
                       "actions": f"U(-{sc['act']},{sc['act']}), resident in HBM" if A else "none",
                       "l2": "flushed (256 MiB write) between timed steps",
                       "launch": {"lanes_per_env": lanes, "envs_per_block": epb},
                       "parallelism": f"env-sharded x{world_size}, no collective on the step path"},
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) leg")
    ap.add_argument("--envs", type=int, default=0, help="environments per GPU (0: the workload's)")
    ap.add_argument("--scene", choices=["ant", "humanoid", "collision_stress", "sphere_pile"], default="ant")
    ap.add_argument("--broad", type=int, choices=[0, 1, 2], default=None, help="broad phase (default: the world's)")
    ap.add_argument("--narrow", type=int, choices=[0, 1, 2], default=None, help="narrow phase (default: the world's)")
    ap.add_argument("--semantics", choices=["reference", "corrected"], default="reference")
    ap.add_argument("--gather", action="store_true",
                    help="with N > 1: also time the optional NCCL all-gather of the step outputs (not in value)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    return run_ours(args, rank, world_size, local_rank)


if __name__ == "__main__":
    sys.exit(main())
