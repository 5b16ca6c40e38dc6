"""Distil the actor of a ``train.py`` run into a small GRU student.

    python examples/tracking12/distill.py --teacher-dir runs/tracking12 --log-dir runs/tracking12_student

The teacher is the newest checkpoint's actor (an upstream rsl_rl PPO checkpoint works the same way); the student is a
recurrent model trained by behaviour cloning on the states it visits itself.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
# run from a checkout without installing the package: the repository root is two levels up
sys.path.insert(1, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from train import train_cfg  # noqa: E402  (the teacher's architecture)

from tt_rsl_rl_b200.env.classic import Tracking12  # noqa: E402
from tt_rsl_rl_b200.runners import DistillationRunner, latest_checkpoint  # noqa: E402


def distill_cfg(engine: str = "auto") -> dict:
    teacher = dict(train_cfg()["actor"])
    student = {"class_name": "RNNModel", "rnn_type": "gru", "rnn_hidden_dim": 64, "hidden_dims": [64],
               "activation": "elu", "obs_normalization": True,
               "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 0.1}}
    return {
        "num_steps_per_env": 24,
        "save_interval": 50,
        "obs_groups": {"student": ["policy"], "teacher": ["policy"]},
        "logger": {"class_name": "CsvLogWriter"},
        "algorithm": {"class_name": "Distillation", "num_learning_epochs": 2, "gradient_length": 12,
                      "learning_rate": 1e-3, "max_grad_norm": 1.0, "loss_type": "mse",
                      "b200_cfg": {"engine": engine}},
        "student": student,
        "teacher": teacher,
    }


def main(argv: list[str] | None = None) -> DistillationRunner:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--teacher-dir", default="runs/tracking12")
    p.add_argument("--log-dir", default="runs/tracking12_student")
    p.add_argument("--envs", type=int, default=4096)
    p.add_argument("--iterations", type=int, default=100)
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--engine", default="auto", choices=["auto", "torch", "cuda"])
    args = p.parse_args(argv)

    teacher = latest_checkpoint(args.teacher_dir)
    if teacher is None:
        raise SystemExit(f"no checkpoint in {args.teacher_dir}")
    torch.manual_seed(args.seed)
    env = Tracking12(args.envs, seed=args.seed, device=args.device)
    runner = DistillationRunner(env, distill_cfg(args.engine), log_dir=args.log_dir, device=args.device)
    if runner.resume_latest() is None:  # a fresh run: the teacher comes from the RL checkpoint
        runner.load(teacher)
    runner.learn(num_learning_iterations=args.iterations, init_at_random_ep_len=True)
    return runner


if __name__ == "__main__":
    main()
