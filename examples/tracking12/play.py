"""Evaluate a run of ``train.py`` and export its policy.

    python examples/tracking12/play.py --log-dir runs/tracking12 --export runs/tracking12/exported

Loads the newest ``model_<it>.pt`` of the run (an upstream rsl_rl checkpoint of the same configuration loads the same
way), runs the deterministic policy on fresh environments and prints the return and length of the episodes that end.
``--export`` writes a TorchScript policy (``policy.pt``) that needs neither this package nor rsl_rl to run.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from train import train_cfg  # noqa: E402  (the configuration the run was trained with)

from tt_rsl_rl_b200.env.classic import Tracking12  # noqa: E402
from tt_rsl_rl_b200.runners import OnPolicyRunner  # noqa: E402
from tt_rsl_rl_b200.runners.play import evaluate  # noqa: E402


def main(argv: list[str] | None = None) -> dict:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--log-dir", default="runs/tracking12")
    p.add_argument("--envs", type=int, default=256)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--export", default=None, help="directory for the TorchScript policy")
    args = p.parse_args(argv)

    env = Tracking12(args.envs, seed=args.seed, device=args.device)
    runner = OnPolicyRunner(env, train_cfg(engine="torch"), log_dir=None, device=args.device)
    path = runner.resume_latest(args.log_dir)
    if path is None:
        raise SystemExit(f"no checkpoint in {args.log_dir}")
    stats = {"checkpoint": path, **evaluate(runner.get_inference_policy(args.device), env, args.steps)}
    if args.export:
        runner.export_policy_to_jit(args.export)
        stats["exported"] = os.path.join(args.export, "policy.pt")
    print(json.dumps(stats))
    return stats


if __name__ == "__main__":
    main()
