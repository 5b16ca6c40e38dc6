"""Evaluate a checkpoint: load a trained policy and run it on an environment, reporting the returns and lengths of the
episodes that finished, or export it.

::

    python -m tt_rsl_rl_b200.runners.play --run-dir logs/run --env cartpole --num-envs 256 --steps 1000
    python -m tt_rsl_rl_b200.runners.play --run-dir logs/run --env my_pkg.envs:make --export-jit exported/

The training configuration is read from ``<run dir>/config.json`` (written by the CSV log writer) or given with
``--cfg``; the newest ``model_<iteration>.pt`` of the run is loaded unless ``--checkpoint`` names one. The reference
plugin's example has the same role for its G1 demo (``examples/g1_walk/play.py``); rendering is not part of this one.
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def evaluate(policy, env, steps: int) -> dict:
    """Run ``policy`` (observations -> actions) for ``steps`` steps; statistics of the episodes that ended."""
    obs = env.get_observations()
    ret = torch.zeros(env.num_envs)
    length = torch.zeros(env.num_envs)
    returns, lengths = [], []
    with torch.inference_mode():
        if hasattr(policy, "reset"):
            policy.reset()
        for _ in range(steps):
            obs, rew, dones, _ = env.step(policy(obs))
            ret += rew.float().cpu().view(-1)
            length += 1
            done = dones.cpu().view(-1) > 0
            if bool(done.any()):
                returns += ret[done].tolist()
                lengths += length[done].tolist()
                ret[done] = 0.0
                length[done] = 0.0
                if hasattr(policy, "reset"):
                    policy.reset(done.to(obs.device if hasattr(obs, "device") else "cpu"))
    mean = (lambda xs: sum(xs) / len(xs) if xs else None)
    return {"episodes": len(returns), "mean_return": mean(returns), "mean_length": mean(lengths),
            "unfinished_mean_return": float(ret.mean())}


def _env(spec: str, num_envs: int, seed: int, device: str):
    from ..env.classic import ENV_CLASSES, make_env

    if spec in ENV_CLASSES:
        return make_env(spec, num_envs, seed=seed, device=device)
    from ..utils.utils import resolve_callable

    return resolve_callable(spec)(num_envs=num_envs, device=device)


def main(argv=None) -> int:
    from . import OnPolicyRunner, latest_checkpoint

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--run-dir", required=True)
    ap.add_argument("--env", required=True, help="a test environment name or 'module:callable(num_envs, device)'")
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--cfg", default=None, help="training configuration (JSON); default: <run dir>/config.json")
    ap.add_argument("--num-envs", type=int, default=256)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--seed", type=int, default=123)
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--export-jit", default=None, help="also write the scripted policy into this folder")
    args = ap.parse_args(argv)
    cfg_path = args.cfg or os.path.join(args.run_dir, "config.json")
    with open(cfg_path) as f:
        cfg = json.load(f)
    cfg = cfg.get("train_cfg", cfg)
    # evaluation runs the actor only: the training extensions (their stored settings are already resolved against the
    # training environment) are left out
    for key in ("rnd_cfg", "symmetry_cfg"):
        cfg.get("algorithm", {}).pop(key, None)
    ckpt = args.checkpoint or latest_checkpoint(args.run_dir)
    if ckpt is None:
        raise SystemExit(f"no model_<iteration>.pt in {args.run_dir}")
    env = _env(args.env, args.num_envs, args.seed, args.device)
    runner = OnPolicyRunner(env, cfg, log_dir=None, device=args.device)
    runner.load(ckpt, map_location=args.device)
    if args.export_jit:
        runner.export_policy_to_jit(args.export_jit)
    stats = evaluate(runner.get_inference_policy(args.device), env, args.steps)
    print(json.dumps({"checkpoint": ckpt, **stats}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
