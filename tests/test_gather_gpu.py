"""The optional output gather over NCCL (zeno_b200.gather) on two GPUs: one process and
one Ant world per GPU, sharded as bench.py shards them; every rank's all-gather must hold
each rank's own observations / rewards / dones at that rank's global env offset, and a
gather to rank 0 the same.  Skipped with fewer than two GPUs (the host logic runs on CPU
in test_multiproc_gloo.py)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
E, WORLD, STEPS = 64, 2, 6
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_dir):
    sys.path.insert(0, str(ROOT))
    from datetime import timedelta
    import torch.distributed as dist
    import bench
    from zeno_b200 import ZenoWorld, scenes
    from zeno_b200.gather import OutputGather
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    w = ZenoWorld(mjcf_string=scenes.ant(), num_envs=E, substeps=4)
    w.set_task(body=1, z_min=0.2, z_max=1.0, auto_reset=True, noise=0.1, seed=5,
               env_offset=bench.shard_env_offset(rank, E))
    rng = np.random.default_rng(10 + rank)
    for _ in range(STEPS):
        w.step(rng.uniform(-1, 1, (E, w.action_dim)).astype(np.float32))
    g = OutputGather.for_world(w)
    allg = [t.cpu().numpy() for t in g.all_gather()]
    to0 = g.gather(dst=0)
    to0 = None if to0 is None else [t.cpu().numpy() for t in to0]
    np.savez(Path(out_dir) / f"rank{rank}.npz", own_obs=w.get_observations(), own_rew=w.get_rewards(),
             own_don=w.get_dones(), all_obs=allg[0], all_rew=allg[1], all_don=allg[2],
             to0=np.array(to0 is not None),
             **({"g_obs": to0[0], "g_rew": to0[1], "g_don": to0[2]} if to0 is not None else {}))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(300)
def test_nccl_gather_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    r = [np.load(tmp_path / f"rank{k}.npz") for k in range(WORLD)]
    for k in range(WORLD):
        sl = slice(k * E, (k + 1) * E)
        for own, full in (("own_obs", "all_obs"), ("own_rew", "all_rew"), ("own_don", "all_don")):
            for j in range(WORLD):  # every rank's all-gather holds rank k's outputs at its offset
                assert np.array_equal(r[j][full][sl], r[k][own]), (own, j, k)
    assert bool(r[0]["to0"]) and not bool(r[1]["to0"])
    for a, b in (("g_obs", "all_obs"), ("g_rew", "all_rew"), ("g_don", "all_don")):
        assert np.array_equal(r[0][a], r[0][b])
