"""PPO on the 12-D tracking task: an actor that sees tracking errors, a critic that also sees the target's private state.

    python examples/tracking12/train.py --device cuda:0 --envs 4096 --iterations 300
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 examples/tracking12/train.py --envs 4096
    python examples/tracking12/train.py --device cpu --envs 256 --iterations 50          # no GPU

A restarted run (same ``--log-dir``) continues from its newest checkpoint. The configuration is plain rsl_rl 5.x; the
only backend-specific part is the optional ``b200_cfg`` dictionary, which can be left out.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

# run from a checkout without installing the package: the repository root is two levels up
sys.path.insert(1, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from tt_rsl_rl_b200.env.classic import Tracking12  # noqa: E402
from tt_rsl_rl_b200.runners import OnPolicyRunner  # noqa: E402


def train_cfg(save_interval: int = 50, engine: str = "auto") -> dict:
    mlp = {"class_name": "MLPModel", "hidden_dims": [256, 128, 64], "activation": "elu", "obs_normalization": True}
    return {
        "num_steps_per_env": 24,
        "save_interval": save_interval,
        "obs_groups": {"actor": ["policy"], "critic": ["policy", "privileged"]},
        "logger": {"class_name": "CsvLogWriter"},
        "algorithm": {
            "class_name": "PPO", "num_learning_epochs": 5, "num_mini_batches": 4, "learning_rate": 1e-3,
            "schedule": "adaptive", "desired_kl": 0.01, "gamma": 0.99, "lam": 0.95, "entropy_coef": 0.005,
            "clip_param": 0.2, "max_grad_norm": 1.0,
            "b200_cfg": {"engine": engine},
        },
        "actor": {**mlp, "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": dict(mlp),
    }


def main(argv: list[str] | None = None) -> OnPolicyRunner:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--envs", type=int, default=4096, help="environments per process")
    p.add_argument("--iterations", type=int, default=300)
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--log-dir", default="runs/tracking12")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--save-interval", type=int, default=50)
    p.add_argument("--engine", default="auto", choices=["auto", "torch", "cuda"])
    args = p.parse_args(argv)

    device = args.device
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and device.startswith("cuda"):
        device = f"cuda:{local_rank}"  # one process per GPU; the runner joins the process group
    seed = args.seed + int(os.environ.get("RANK", "0"))  # different environments on every rank
    torch.manual_seed(seed)

    env = Tracking12(args.envs, seed=seed, device=device)
    runner = OnPolicyRunner(env, train_cfg(args.save_interval, args.engine), log_dir=args.log_dir, device=device)
    resumed = runner.resume_latest()
    if resumed and local_rank == 0:
        print(f"resuming from {resumed}")
    runner.learn(num_learning_iterations=args.iterations, init_at_random_ep_len=True)  # saves model_<last>.pt at the end
    return runner


if __name__ == "__main__":
    main()
