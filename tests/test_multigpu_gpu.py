"""Data-parallel engine on 2+ GPUs: one process per GPU (NCCL bootstrap, CUDA-IPC peer exchange).

Checks that replicas trained on different rollouts stay bit-identical (rank-ordered peer reduction), that the
normaliser statistics are global, and that the parameter broadcast makes every rank start from rank 0's weights.
Skipped when fewer than two GPUs are visible.
"""

import json
import os
import socket
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                         timeout=datetime.timedelta(seconds=60))
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    torch.manual_seed(100 + rank)  # different initial weights per rank: the broadcast must fix them
    cfg = {
        "num_steps_per_env": 8, "save_interval": 1000, "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "algorithm": {"class_name": "PPO", "num_learning_epochs": 2, "num_mini_batches": 2,
                      "b200_cfg": {"comm_timeout_ms": 20000}},
        "actor": {"class_name": "MLPModel", "hidden_dims": [128, 64], "obs_normalization": True,
                  "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": [128, 64], "obs_normalization": True},
    }
    env = LinearGaussianVecEnv(512, obs_dim=48, num_actions=12, privileged_dim=3, device=f"cuda:{rank}",
                               seed=10 + rank)
    runner = OnPolicyRunner(env, cfg, log_dir=None, device=f"cuda:{rank}")
    assert runner.alg.engine is not None and runner.alg.engine.comm is not None
    runner.learn(3)
    eng = runner.alg.engine
    flat = eng.flat.double()
    norm = runner.alg.actor.obs_normalizer
    res = {
        "rank": rank,
        "checksum": float(flat.sum()),
        "hash": float((flat * torch.arange(flat.numel(), device=flat.device, dtype=torch.float64).sin()).sum()),
        "count": int(norm.count),
        "mean0": float(norm._mean.view(-1)[0]),
        "status": eng.status.tolist(),
        "lr": runner.alg.learning_rate,
    }
    gathered = [torch.zeros_like(eng.flat) for _ in range(world)]
    torch.distributed.all_gather(gathered, eng.flat)
    res["identical"] = all(torch.equal(gathered[0], g) for g in gathered)
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_data_parallel_replicas_bit_identical():
    world = min(torch.cuda.device_count(), 4)
    out_dir = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_worker, args=(world, _free_port(), out_dir), nprocs=world, join=True)
    res = [json.load(open(os.path.join(out_dir, f"rank{r}.json"))) for r in range(world)]
    assert all(r["identical"] for r in res)
    assert all(r["status"][0] == 0 for r in res)
    assert len({r["hash"] for r in res}) == 1
    # global normaliser statistics: 3 updates x T*N rows on every rank
    assert all(r["count"] == 3 * 8 * 512 * world for r in res)
    assert len({r["mean0"] for r in res}) == 1
    assert len({r["lr"] for r in res}) == 1
