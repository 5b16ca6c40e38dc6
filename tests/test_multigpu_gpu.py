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


def _mirror(env=None, obs=None, actions=None):
    """Two-copy signed-permutation augmentation (reversal of every group, sign flip of odd columns)."""
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    def m(x):
        d = x.shape[1]
        sign = torch.ones(d, device=x.device)
        sign[1::2] = -1.0
        return x.flip(1) * sign

    out_obs = None if obs is None else TensorDict({g: torch.cat([obs[g], m(obs[g])]) for g in obs.keys()},
                                                  batch_size=[2 * obs.batch_size[0]], device=obs.device)
    out_act = None if actions is None else torch.cat([actions, m(actions)])
    return out_obs, out_act


def _cfg(kind: str) -> dict:
    mlp = lambda extra: dict({"class_name": "MLPModel", "hidden_dims": [128, 64], "obs_normalization": True}, **extra)
    dist = {"distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}}
    alg = {"class_name": "PPO", "num_learning_epochs": 2, "num_mini_batches": 2,
           "b200_cfg": {"comm_timeout_ms": 20000, "engine": "cuda"}}
    cfg = {"num_steps_per_env": 8, "save_interval": 1000, "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
           "algorithm": alg, "actor": mlp(dist), "critic": mlp({})}
    if kind == "rnd_sym":
        cfg["obs_groups"]["rnd_state"] = ["critic"]
        alg["rnd_cfg"] = {"num_outputs": 8, "predictor_hidden_dims": [64], "target_hidden_dims": [64], "weight": 0.5,
                          "state_normalization": True}
        alg["symmetry_cfg"] = {"data_augmentation_func": _mirror, "use_data_augmentation": True,
                               "use_mirror_loss": True, "mirror_loss_coeff": 1.0}
    elif kind in ("gru", "lstm", "gru_rnd"):
        for k in ("actor", "critic"):
            cfg[k].update({"class_name": "RNNModel", "rnn_type": kind[:4].rstrip("_"), "rnn_hidden_dim": 64})
        if kind == "gru_rnd":
            cfg["obs_groups"]["rnd_state"] = ["critic"]
            alg["rnd_cfg"] = {"num_outputs": 8, "predictor_hidden_dims": [64], "target_hidden_dims": [64],
                              "weight": 0.5, "state_normalization": True}
    elif kind == "distill_rnn":
        cfg = {"num_steps_per_env": 8, "save_interval": 1000,
               "obs_groups": {"student": ["policy"], "teacher": ["critic"]},
               "algorithm": {"class_name": "Distillation", "num_learning_epochs": 2, "gradient_length": 3,
                             "b200_cfg": {"comm_timeout_ms": 20000, "engine": "cuda"}},
               "student": dict(mlp(dist), class_name="RNNModel", rnn_type="gru", rnn_hidden_dim=64),
               "teacher": dict(mlp({}), class_name="RNNModel", rnn_type="lstm", rnn_hidden_dim=64)}
    elif kind == "distill":
        cfg = {"num_steps_per_env": 8, "save_interval": 1000,
               "obs_groups": {"student": ["policy"], "teacher": ["critic"]},
               "algorithm": {"class_name": "Distillation", "num_learning_epochs": 1, "gradient_length": 2,
                             "b200_cfg": {"comm_timeout_ms": 20000, "engine": "cuda"}},
               "student": mlp(dist), "teacher": mlp({})}
    return cfg


def _worker(rank: int, world: int, port: int, out_dir: str, kind: str = "mlp") -> None:
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                         timeout=datetime.timedelta(seconds=60))
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv
    from tt_rsl_rl_b200.runners import DistillationRunner, OnPolicyRunner

    torch.manual_seed(100 + rank)  # different initial weights per rank: the broadcast must fix them
    cfg = _cfg(kind)
    env = LinearGaussianVecEnv(512, obs_dim=48, num_actions=12, privileged_dim=3, device=f"cuda:{rank}",
                               seed=10 + rank, reset_prob=0.02)
    runner_cls = DistillationRunner if kind.startswith("distill") else OnPolicyRunner
    runner = runner_cls(env, cfg, log_dir=None, device=f"cuda:{rank}")
    if kind.startswith("distill"):
        runner.alg.teacher_loaded = True
    assert runner.alg.engine is not None and runner.alg.engine.comm is not None
    runner.learn(3)
    eng = runner.alg.engine
    flat = eng.flat.double()
    norm = (runner.alg.student if kind.startswith("distill") else runner.alg.actor).obs_normalizer
    res = {
        "rank": rank,
        "checksum": float(flat.sum()),
        "hash": float((flat * torch.arange(flat.numel(), device=flat.device, dtype=torch.float64).sin()).sum()),
        "count": int(norm.count),
        "mean0": float(norm._mean.view(-1)[0]),
        "status": eng.status.tolist(),
        "lr": runner.alg.learning_rate,
    }
    if kind.startswith("distill"):  # the frozen teacher must be rank 0's on every rank
        res["teacher"] = float(sum(p.double().sum() for p in runner.alg.teacher.parameters()))
    if kind in ("rnd_sym", "gru_rnd"):
        res["rnd_target"] = float(sum(p.double().sum() for p in runner.alg.rnd.target.parameters()))
        res["rnd_count"] = int(runner.alg.rnd.state_normalizer.count)
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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kind", ["rnd_sym", "gru", "lstm", "gru_rnd", "distill", "distill_rnn"])
def test_data_parallel_engines_bit_identical(kind):
    world = 2
    out_dir = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_worker, args=(world, _free_port(), out_dir, kind), nprocs=world, join=True)
    res = [json.load(open(os.path.join(out_dir, f"rank{r}.json"))) for r in range(world)]
    assert all(r["identical"] for r in res), kind
    assert all(r["status"][0] == 0 for r in res)
    assert all(r["count"] == 3 * 8 * 512 * world for r in res)
    assert len({r["mean0"] for r in res}) == 1
    for key in ("teacher", "rnd_target", "rnd_count"):
        if key in res[0]:
            assert len({r[key] for r in res}) == 1, key
