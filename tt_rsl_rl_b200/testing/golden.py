"""Golden learning curves of the seeded test environments and the acceptance rule applied to them.

The golden curves are recorded with the upstream rsl_rl runner on the CPU (:func:`record`, one CSV per environment and
seed plus ``summary.json``). A run of this framework passes on an environment when the mean over its seeds of the final
reward (mean of ``Train/mean_reward`` over the last ``FINAL_WINDOW`` iterations) is finite and at least

    golden mean - max(golden std over seeds, 5 % of |golden mean|).

The reference plugin applies the same rule to its own golden runs (``rsl_rl_tt/testing/golden.py:28-60``).

Command line::

    python -m tt_rsl_rl_b200.testing.golden record --envs cartpole pendulum --seeds 0 1 2
    python -m tt_rsl_rl_b200.testing.golden summarize --envs cartpole     # statistics from the CSVs in place
    python -m tt_rsl_rl_b200.testing.golden check --envs cartpole --seeds 0 1 2 --device cuda:0
    python -m tt_rsl_rl_b200.testing.golden tb2csv --tb-dir logs/rsl_rl/cartpole/<run> --out gpu_seed0.csv
    python -m tt_rsl_rl_b200.testing.golden compare --ref gpu_seed0.csv gpu_seed1.csv --run a/metrics.csv b/metrics.csv

The last two compare any run logged by TensorBoard (an upstream run on a GPU, for instance) with this framework's runs
under the same rule, as the reference plugin does for its own runs (``scripts/tb_to_csv.py``,
``scripts/compare_curves.py``).
"""

from __future__ import annotations

import argparse
import csv
import json
import math
import os
import statistics
import sys
import tempfile
from pathlib import Path

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
FINAL_WINDOW = 10
SEEDS = (0, 1, 2)
# tracking's final reward varies more between runs (a change of summation order alone moves it by +-10), so its
# golden statistics use five seeds
ENV_SEEDS = {"tracking12": (0, 1, 2, 3, 4)}
REWARD = "Train/mean_reward"
# columns kept in the committed curves
KEEP = ("iteration", "Train/mean_reward", "Train/mean_episode_length", "Loss/value", "Loss/surrogate", "Loss/entropy",
        "Loss/learning_rate", "Policy/mean_std")


def seeds_for(env_name: str) -> tuple[int, ...]:
    """The seeds of an environment's golden curves."""
    return ENV_SEEDS.get(env_name, SEEDS)


def read_curve(path: str | Path) -> list[dict[str, float | None]]:
    """Rows of a metrics CSV; empty cells become ``None``."""
    with open(path, newline="") as f:
        return [{k: (float(v) if v not in ("", None) else None) for k, v in row.items()} for row in csv.DictReader(f)]


def write_curve(path: str | Path, rows: list[dict], columns=KEEP) -> None:
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(columns), extrasaction="ignore", restval="")
        w.writeheader()
        for r in rows:
            w.writerow({k: ("" if r.get(k) is None else r[k]) for k in columns})


def final_reward(rows: list[dict], window: int = FINAL_WINDOW) -> float:
    """Mean of the last ``window`` logged rewards (NaN when the run never finished an episode)."""
    vals = [r[REWARD] for r in rows if r.get(REWARD) is not None][-window:]
    return statistics.mean(vals) if vals else float("nan")


def threshold(mean: float, std: float) -> float:
    """Lowest passing final reward for golden seeds of mean ``mean`` and standard deviation ``std``."""
    return mean - max(std, 0.05 * abs(mean))


def summarize(finals: list[float]) -> dict:
    return {"final_rewards": finals, "final_reward_mean": statistics.mean(finals),
            "final_reward_std": statistics.stdev(finals) if len(finals) > 1 else 0.0}


def load_summary(golden_dir: str | Path = GOLDEN_DIR) -> dict:
    return json.loads((Path(golden_dir) / "summary.json").read_text())


def verdict(env_name: str, finals: list[float], curves_finite: bool = True, summary: dict | None = None) -> dict:
    """Apply the acceptance rule to the final rewards of a run's seeds."""
    ref = (summary or load_summary())["envs"][env_name]
    thr = threshold(ref["final_reward_mean"], ref["final_reward_std"])
    finite = curves_finite and bool(finals) and all(math.isfinite(x) for x in finals)
    mean = statistics.mean(finals) if finals else float("nan")
    return {"env": env_name, "final_rewards": finals, "mean": mean, "golden_mean": ref["final_reward_mean"],
            "golden_std": ref["final_reward_std"], "threshold": thr, "all_finite": finite,
            "passes": bool(finite and mean >= thr)}


def _curve_finite(rows: list[dict]) -> bool:
    return all(v is None or math.isfinite(v) for r in rows for v in r.values())


def record(envs, seeds=None, out_dir: str | Path = GOLDEN_DIR, iterations: int | None = None,
           num_threads: int | None = None) -> dict:
    """Train every environment with upstream rsl_rl on the CPU and write the curves and ``summary.json``."""
    from .reference import SPECS, train

    out_dir = Path(out_dir)
    summary_path = out_dir / "summary.json"
    summary = json.loads(summary_path.read_text()) if summary_path.exists() else {"envs": {}}
    summary.update({"final_window": FINAL_WINDOW, "impl": "upstream rsl_rl (CPU)"})
    for env_name in envs:
        (out_dir / env_name).mkdir(parents=True, exist_ok=True)
        finals, runs = [], []
        env_seeds = seeds_for(env_name) if seeds is None else tuple(seeds)
        for seed in env_seeds:
            with tempfile.TemporaryDirectory() as tmp:
                info = train(env_name, seed, tmp, impl="upstream", iterations=iterations, num_threads=num_threads)
                rows = read_curve(os.path.join(tmp, "metrics.csv"))
            write_curve(out_dir / env_name / f"seed{seed}.csv", rows)
            finals.append(final_reward(rows))
            runs.append({"seed": seed, "wall_s": round(info["wall_s"], 1), "iterations": info["iterations"],
                         "num_threads": info["num_threads"]})  # the thread count sets the matmul summation order
        spec = SPECS[env_name]
        summary["envs"][env_name] = {**summarize(finals), "seeds": list(env_seeds), "runs": runs,
                                     "num_envs": spec.num_envs, "num_steps": spec.num_steps,
                                     "hidden": list(spec.hidden)}
        summary_path.write_text(json.dumps(summary, indent=1))
    return summary


def summarize_dir(envs, seeds=None, golden_dir: str | Path = GOLDEN_DIR) -> dict:
    """Rebuild the final-reward statistics of ``summary.json`` from the curves already in ``golden_dir`` (per-run
    metadata recorded earlier is kept)."""
    from .reference import SPECS

    golden_dir = Path(golden_dir)
    path = golden_dir / "summary.json"
    summary = json.loads(path.read_text()) if path.exists() else {"envs": {}}
    summary.update({"final_window": FINAL_WINDOW, "impl": "upstream rsl_rl (CPU)"})
    for env_name in envs:
        env_seeds = seeds_for(env_name) if seeds is None else tuple(seeds)
        finals = [final_reward(read_curve(golden_dir / env_name / f"seed{s}.csv")) for s in env_seeds]
        spec = SPECS[env_name]
        prev = summary["envs"].get(env_name, {})
        summary["envs"][env_name] = {**prev, **summarize(finals), "seeds": list(env_seeds), "num_envs": spec.num_envs,
                                     "num_steps": spec.num_steps, "hidden": list(spec.hidden),
                                     "iterations": spec.iterations}
    path.write_text(json.dumps(summary, indent=1))
    return summary


def check(envs, seeds=None, device: str = "cpu", iterations: int | None = None, log_root: str | None = None,
          golden_dir: str | Path = GOLDEN_DIR, num_threads: int | None = None, engine: str | None = None,
          mixed_precision: bool = False) -> list[dict]:
    """Train every environment with this framework on ``device`` and apply the acceptance rule. ``engine`` selects
    the execution path (``"cuda"`` fused engines, ``"torch"`` the PyTorch path; default: automatic)."""
    from .reference import train

    summary = load_summary(golden_dir)
    out = []
    for env_name in envs:
        finals, finite = [], True
        for seed in (seeds_for(env_name) if seeds is None else seeds):
            with tempfile.TemporaryDirectory() as tmp:
                log_dir = os.path.join(log_root, env_name, f"seed{seed}") if log_root else tmp
                train(env_name, seed, log_dir, impl="b200", device=device, iterations=iterations,
                      num_threads=num_threads, engine=engine, mixed_precision=mixed_precision)
                rows = read_curve(os.path.join(log_dir, "metrics.csv"))
            finals.append(final_reward(rows))
            finite &= _curve_finite(rows)
        out.append(verdict(env_name, finals, finite, summary))
    return out


def tb_to_csv(run_dir: str | Path, out: str | Path) -> int:
    """Scalars of the TensorBoard event files under ``run_dir`` (the default writer of a run, e.g. an Isaac Lab GPU
    run) as a CSV of this package's layout: ``iteration`` then one column per tag. Returns the number of rows."""
    from tensorboard.backend.event_processing.event_accumulator import EventAccumulator

    acc = EventAccumulator(str(run_dir), size_guidance={"scalars": 0})  # 0: keep every event
    acc.Reload()
    tags = [t for t in acc.Tags()["scalars"] if not t.endswith("/time")]
    if not tags:
        raise ValueError(f"no scalar events under {run_dir}")
    table: dict[int, dict[str, float]] = {}
    for tag in tags:
        for ev in acc.Scalars(tag):
            table.setdefault(int(ev.step), {"iteration": int(ev.step)})[tag] = float(ev.value)
    rows = [table[k] for k in sorted(table)]
    write_curve(out, rows, columns=["iteration", *tags])
    return len(rows)


def compare_runs(reference: list[str | Path], runs: list[str | Path]) -> dict:
    """The acceptance rule between two sets of curves (CSV files; e.g. a GPU reference run converted with
    :func:`tb_to_csv` against this framework's runs). With one reference seed only the 5 % margin applies."""
    ref_finals = [final_reward(read_curve(p)) for p in reference]
    run_curves = [read_curve(p) for p in runs]
    summary = {"envs": {"runs": summarize(ref_finals)}}
    return verdict("runs", [final_reward(c) for c in run_curves], all(_curve_finite(c) for c in run_curves), summary)


def stability(rows: list[dict], reach: float = 499.0, collapse: float = 450.0) -> dict:
    """Whether a run that reached ``reach`` (cart-pole's maximum) later fell below ``collapse``: the first iteration
    at the level, the lowest reward after it and the final reward (the reference plugin's stability study has the
    same measures: ``scripts/stability_cartpole.py``)."""
    rewards = [(r["iteration"], r[REWARD]) for r in rows if r.get(REWARD) is not None]
    first = next((it for it, v in rewards if v >= reach), None)
    after = [v for it, v in rewards if first is not None and it >= first]
    low = min(after) if after else None
    return {"first_at_level": first, "min_after": low, "final": final_reward(rows),
            "collapsed": bool(low is not None and low < collapse)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("mode", choices=("record", "summarize", "check", "compare", "tb2csv"))
    ap.add_argument("--ref", nargs="+", default=None, help="compare: reference curves (CSV)")
    ap.add_argument("--run", nargs="+", default=None, help="compare: curves of the run under test (CSV)")
    ap.add_argument("--tb-dir", default=None, help="tb2csv: folder with TensorBoard event files")
    ap.add_argument("--out", default=None, help="tb2csv: CSV to write")
    ap.add_argument("--envs", nargs="+", default=["cartpole", "pendulum", "tracking12", "cartpole_po"])
    ap.add_argument("--seeds", nargs="+", type=int, default=None, help="default: the environment's golden seeds")
    ap.add_argument("--device", default="cpu", help="check only: device of this framework's run")
    ap.add_argument("--iterations", type=int, default=None, help="override the spec's iteration count")
    ap.add_argument("--threads", type=int, default=None)
    ap.add_argument("--golden-dir", default=str(GOLDEN_DIR))
    ap.add_argument("--log-root", default=None, help="check only: keep the curves of the run under this folder")
    ap.add_argument("--engine", choices=("auto", "cuda", "torch"), default=None,
                    help="check only: execution path of this framework (fused engines or the PyTorch path)")
    ap.add_argument("--mixed-precision", action="store_true", help="check only: bf16 autocast on the PyTorch path")
    args = ap.parse_args(argv)
    if args.mode == "record":
        print(json.dumps(record(args.envs, args.seeds, args.golden_dir, args.iterations, args.threads), indent=1))
        return 0
    if args.mode == "summarize":
        print(json.dumps(summarize_dir(args.envs, args.seeds, args.golden_dir), indent=1))
        return 0
    if args.mode == "tb2csv":
        if not (args.tb_dir and args.out):
            ap.error("tb2csv needs --tb-dir and --out")
        print(json.dumps({"rows": tb_to_csv(args.tb_dir, args.out), "out": args.out}))
        return 0
    if args.mode == "compare":
        if not (args.ref and args.run):
            ap.error("compare needs --ref and --run")
        result = compare_runs(args.ref, args.run)
        print(json.dumps(result))
        return 0 if result["passes"] else 1
    results = check(args.envs, args.seeds, args.device, args.iterations, args.log_root, args.golden_dir, args.threads,
                    engine=args.engine, mixed_precision=args.mixed_precision)
    for r in results:
        print(json.dumps(r))
    return 0 if all(r["passes"] for r in results) else 1


if __name__ == "__main__":
    sys.exit(main())
