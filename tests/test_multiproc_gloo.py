"""Multi-process host logic (world size 2, gloo on CPU): environments sharded across
ranks with bench.py's offsets must give the same per-env results as one process owning
all envs (the reset-noise stream is keyed by the global env index), and the max-over-ranks
timing reduction must return the slowest rank, and the optional output gather must
deliver every rank's observations / rewards / dones in global env order.  The physics here
is the CPU oracle, so the test needs no GPU; the GPU path shards identically (bench.py uses
the same helpers; zeno_b200.gather runs over NCCL there)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
E_PER_RANK, WORLD, STEPS = 4, 2, 40


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene_and_actions():
    sys.path.insert(0, str(ROOT))
    from zeno_b200 import scenes
    xml = scenes.ant()
    acts = np.random.default_rng(99).uniform(-1, 1, size=(STEPS, E_PER_RANK * WORLD, 8)).astype(np.float32)
    return xml, acts


def _rank_main(rank, port, out_dir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch.distributed as dist
    import bench
    from oracle.zeno_oracle import OracleWorld
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    xml, acts = _scene_and_actions()
    off = bench.shard_env_offset(rank, E_PER_RANK)
    o = OracleWorld(xml, num_envs=E_PER_RANK, substeps=4)
    o.set_task(body=1, z_min=0.2, z_max=1.0, auto_reset=True, noise=0.1, seed=3, env_offset=off)
    for s in range(STEPS):
        o.step(acts[s, off:off + E_PER_RANK])
    st = o.state()
    np.savez(Path(out_dir) / f"rank{rank}.npz", **{k: st[k] for k in ("positions", "dones", "contact_counts")})
    slowest = bench.reduce_max(float(rank + 1) * 0.5, dist, "cpu")
    assert slowest == WORLD * 0.5
    import torch
    from zeno_b200.gather import OutputGather
    g = OutputGather(torch.from_numpy(st["observations"]), torch.from_numpy(st["rewards"]),
                     torch.from_numpy(st["dones"]))
    allg = [t.numpy().copy() for t in g.all_gather()]
    to1 = g.gather(dst=1)
    assert (to1 is None) == (rank != 1)
    if to1 is not None:
        assert all(np.array_equal(a, t.numpy()) for a, t in zip(allg, to1))
    np.savez(Path(out_dir) / f"gather{rank}.npz", obs=allg[0], rewards=allg[1], dones=allg[2])
    with pytest.raises(ValueError):  # shapes differ across ranks: every rank refuses
        OutputGather(torch.zeros((rank + 1, 3)), torch.zeros(rank + 1), torch.zeros(rank + 1, dtype=torch.uint8))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_oracle_matches_single_process(tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(port, str(tmp_path)), nprocs=WORLD, join=True)
    from oracle.zeno_oracle import OracleWorld
    xml, acts = _scene_and_actions()
    o = OracleWorld(xml, num_envs=E_PER_RANK * WORLD, substeps=4)
    o.set_task(body=1, z_min=0.2, z_max=1.0, auto_reset=True, noise=0.1, seed=3, env_offset=0)
    resets = 0
    for s in range(STEPS):
        o.step(acts[s])
        resets += int(o.state()["dones"].sum())
    full = o.state()
    assert resets > 0  # resets happened, so the noise keying is exercised
    for r in range(WORLD):
        part = np.load(tmp_path / f"rank{r}.npz")
        sl = slice(r * E_PER_RANK, (r + 1) * E_PER_RANK)
        for k in ("positions", "dones", "contact_counts"):
            assert np.array_equal(np.ascontiguousarray(part[k]).view(np.uint8),
                                  np.ascontiguousarray(full[k][sl]).view(np.uint8)), k
        g = np.load(tmp_path / f"gather{r}.npz")
        for k, ref in (("obs", full["observations"]), ("rewards", full["rewards"]), ("dones", full["dones"])):
            assert np.array_equal(g[k].view(np.uint8), np.ascontiguousarray(ref).view(np.uint8)), k


def _dying_rank_main(rank, port, out_dir):
    """Rank 1 leaves between steps, before the gather; rank 0's gather must end with an
    error within the process group's timeout instead of waiting for good."""
    sys.path.insert(0, str(ROOT))
    import time
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from zeno_b200.gather import OutputGather
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=timedelta(seconds=10))
    g = OutputGather(torch.zeros((4, 3)), torch.zeros(4), torch.zeros(4, dtype=torch.uint8))
    g.all_gather()
    if rank == 1:
        os._exit(0)  # no destroy, no further collective
    t0 = time.monotonic()
    try:
        g.all_gather()
        outcome = "completed"
    except Exception as e:  # gloo reports the closed peer (or the timeout)
        outcome = type(e).__name__
    (Path(out_dir) / "rank0.txt").write_text(f"{outcome} {time.monotonic() - t0:.1f}")
    os._exit(0)


@pytest.mark.timeout(120)
def test_gather_reports_a_rank_that_left(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_dying_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    outcome, secs = (tmp_path / "rank0.txt").read_text().split()
    assert outcome != "completed" and float(secs) < 60
