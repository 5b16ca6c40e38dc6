"""Device time per kernel entry point over one eager PPO iteration (rollout, returns, update) of this framework's
CUDA engine on a null environment, as a table sorted by total time::

    python -m tt_rsl_rl_b200.ops.profile --envs 65536 --hidden 512,256,128

The iteration runs without CUDA graphs (every launch comes from Python and is timed by
:class:`tt_rsl_rl_b200.ops.profile_ops`); one untimed iteration warms up first. The reference plugin's op profiler
has the same role (``scripts/profile_ops.py``).
"""

from __future__ import annotations

import argparse
import json

import torch

from . import profile_ops


def profile_iteration(alg, env, steps: int) -> profile_ops:
    """Time every launching entry point of one rollout + returns + update of ``alg``."""
    obs = env.get_observations()
    with profile_ops() as prof:
        with torch.inference_mode():
            for _ in range(steps):
                actions = alg.act(obs)
                obs, rewards, dones, extras = env.step(actions)
                alg.process_env_step(obs, rewards, dones, extras)
            alg.compute_returns(obs)
        alg.update()
    return prof


def main(argv=None) -> None:
    from ..runners.bench_matrix import build, run_iterations

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--envs", type=int, default=16384)
    ap.add_argument("--hidden", default="512,256,128")
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--mini-batches", type=int, default=4)
    ap.add_argument("--epochs", type=int, default=5)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    hidden = [int(v) for v in args.hidden.split(",")]
    alg, env = build("b200", args.device, args.envs, hidden, args.steps, args.mini_batches, args.epochs,
                     b200_cfg={"graphs": False})
    if getattr(alg, "engine", None) is None:
        raise SystemExit("the CUDA engine is not active for this configuration; nothing to profile")
    run_iterations(alg, env, args.steps, iters=1, warmup=0, device=args.device)  # warm-up
    prof = profile_iteration(alg, env, args.steps)
    rows = prof.table()
    for r in rows:
        print(json.dumps(r))
    print(json.dumps({"total_ms": round(sum(r["total_ms"] for r in rows), 3),
                      "launches": sum(r["calls"] for r in rows)}))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
