"""Algorithm cost per PPO iteration over a grid of environment counts and MLP sizes, with an environment that does no
work (:class:`~tt_rsl_rl_b200.env.null.NullVecEnv`), for this framework or upstream rsl_rl.

Every iteration is split into act / env / process (summed over the rollout's steps), returns and update; with a CUDA
device the phase boundaries synchronise the device, so the split adds a little host latency that the headline
benchmark (``bench.py``, whole iterations timed with CUDA events) does not have. Medians over the timed iterations are
printed as one JSON line per grid point::

    python -m tt_rsl_rl_b200.runners.bench_matrix --device cuda:0 --envs 4096 16384 65536 \
        --hidden 512,256,128 1024,1024,512
    python -m tt_rsl_rl_b200.runners.bench_matrix --impl upstream --envs 4096 --hidden 512,256,128

The reference plugin measures the same split with its matrix benchmark (``scripts/bench_matrix.py:54-114``).
"""

from __future__ import annotations

import argparse
import json
import statistics
import time

import torch

from ..env.null import NullVecEnv

SHAPES = {
    # actor obs, critic obs, actions
    "humanoid": ({"policy": 96, "critic": 99}, 29),
    "tracking12": ({"policy": 36, "critic": 84}, 12),
}


def make_cfg(hidden: list[int], steps: int, mini_batches: int = 4, epochs: int = 5) -> dict:
    mlp = {"class_name": "MLPModel", "hidden_dims": list(hidden), "activation": "elu", "obs_normalization": True}
    return {
        "num_steps_per_env": steps,
        "save_interval": 10_000,
        "check_for_nan": False,  # a host check of the environment's outputs, not part of the algorithm's cost
        "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "actor": {**mlp, "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": dict(mlp),
        "algorithm": {"class_name": "PPO", "num_learning_epochs": epochs, "num_mini_batches": mini_batches,
                      "learning_rate": 1e-3, "schedule": "adaptive", "desired_kl": 0.01, "entropy_coef": 0.005,
                      "max_grad_norm": 1.0},
    }


def build(impl: str, device: str, num_envs: int, hidden: list[int], steps: int = 24, mini_batches: int = 4,
          epochs: int = 5, shape: str = "humanoid", seed: int = 0, b200_cfg: dict | None = None):
    """``(algorithm, env)`` of a runner of ``impl`` ("b200" or "upstream") on a null environment; ``b200_cfg`` goes
    to this framework's algorithm section."""
    groups, num_actions = SHAPES[shape]
    torch.manual_seed(seed)
    env = NullVecEnv(num_envs, groups, num_actions, seed=seed, device=device)
    cfg = make_cfg(hidden, steps, mini_batches, epochs)
    if b200_cfg and impl == "b200":
        cfg["algorithm"]["b200_cfg"] = dict(b200_cfg)
    if impl == "upstream":
        if torch.device(device).type != "cpu":
            raise ValueError("the upstream runner is measured on the CPU here")
        from ..testing.reference import UpstreamEnvAdapter, upstream_runners

        runner_cls, _, td_cls = upstream_runners()
        runner = runner_cls(UpstreamEnvAdapter(env, td_cls), cfg, log_dir=None, device="cpu")
        return runner.alg, UpstreamEnvAdapter(env, td_cls)
    from .on_policy_runner import OnPolicyRunner

    runner = OnPolicyRunner(env, cfg, log_dir=None, device=device)
    return runner.alg, env


def run_iterations(alg, env, steps: int, iters: int, warmup: int, device: str) -> dict:
    """Median milliseconds of each phase over ``iters`` iterations after ``warmup``; env-steps per second."""
    cuda = torch.device(device).type == "cuda"

    def now() -> float:
        if cuda:
            torch.cuda.synchronize(device)
        return time.perf_counter()

    alg.train_mode()
    obs = env.get_observations()
    rows = []
    for _ in range(warmup + iters):
        t0 = now()
        t_act = t_env = t_proc = 0.0
        with torch.inference_mode():
            for _ in range(steps):
                a0 = now()
                actions = alg.act(obs)
                a1 = now()
                obs, rewards, dones, extras = env.step(actions)
                a2 = now()
                alg.process_env_step(obs, rewards, dones, extras)
                a3 = now()
                t_act, t_env, t_proc = t_act + a1 - a0, t_env + a2 - a1, t_proc + a3 - a2
            r0 = now()
            alg.compute_returns(obs)
            t_ret = now() - r0
        u0 = now()
        alg.update()
        t_upd = now() - u0
        rows.append({"act": t_act, "env": t_env, "process": t_proc, "returns": t_ret, "update": t_upd,
                     "total": now() - t0})
    med = {k: statistics.median(r[k] for r in rows[warmup:]) * 1e3 for k in rows[0]}
    out = {f"{k}_ms": round(v, 3) for k, v in med.items()}
    out["env_steps_per_s"] = round(env.num_envs * steps / (med["total"] / 1e3), 1)
    engine = getattr(alg, "engine", None)
    if engine is not None:
        out["engine"] = type(engine).__name__
    return out


def matrix(impl: str, device: str, envs: list[int], hiddens: list[list[int]], steps: int = 24, iters: int = 3,
           warmup: int = 1, mini_batches: int = 4, epochs: int = 5, shape: str = "humanoid"):
    """Yield one result dict per (num_envs, hidden) point."""
    for hidden in hiddens:
        for n in envs:
            alg, env = build(impl, device, n, hidden, steps, mini_batches, epochs, shape)
            res = run_iterations(alg, env, steps, iters, warmup, device)
            yield {"impl": impl, "device": str(device), "num_envs": n, "hidden": hidden, "num_steps": steps,
                   "mini_batches": mini_batches, "epochs": epochs, "shape": shape, **res}
            del alg, env
            if torch.device(device).type == "cuda":
                torch.cuda.empty_cache()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--impl", choices=("b200", "upstream"), default="b200")
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--envs", type=int, nargs="+", default=[4096, 16384, 65536])
    ap.add_argument("--hidden", nargs="+", default=["512,256,128"], help="comma-separated layer sizes per point")
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--mini-batches", type=int, default=4)
    ap.add_argument("--epochs", type=int, default=5)
    ap.add_argument("--shape", choices=sorted(SHAPES), default="humanoid")
    ap.add_argument("--threads", type=int, default=None, help="torch CPU threads")
    ap.add_argument("--out", default=None, help="also write the results as a JSON list")
    args = ap.parse_args(argv)
    if args.threads:
        torch.set_num_threads(args.threads)
    hiddens = [[int(v) for v in h.split(",")] for h in args.hidden]
    results = []
    for res in matrix(args.impl, args.device, args.envs, hiddens, args.steps, args.iters, args.warmup,
                      args.mini_batches, args.epochs, args.shape):
        print(json.dumps(res), flush=True)
        results.append(res)
    if args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)


if __name__ == "__main__":
    main()
