#!/usr/bin/env python
"""Benchmark: PPO training throughput (samples/s) of one learn() iteration on the headline configuration.

Configuration 1 (the default): 65536 environments in total split evenly across ranks, synthetic
linear-Gaussian environment (actor obs 96, critic obs 99, 29 actions), actor and critic MLPs [512, 256, 128] ELU with
empirical observation normalisation, 24 steps per environment, 5 epochs x 4 minibatches, bf16 GEMM operands with fp32
master weights and Adam. Data: synthetic, seeded; weights: random init.

A step is one ``OnPolicyRunner.learn`` iteration (rollout of 24 env steps, returns, update, normaliser update), driven
through the public API. Timing: W untimed warm-up iterations, then K iterations bracketed by a barrier and
``torch.cuda.synchronize()`` and timed with CUDA events on the launching stream; the max over ranks is reported.
Every iteration streams ~T*N*S*4 bytes of rollout data (the rollout arena alone is far larger than the 126 MB L2),
so consecutive iterations do not run from a warm L2.

``value`` is measured with the environment's process noise generated on the device. ``e2e`` repeats the measurement
with the noise of every environment step copied from pinned host memory (``host_noise=True``) plus the device-to-host
read of each iteration's loss statistics and learning rate.

Usage: ``python bench.py --gpus N --steps K --warmup W [--impl ours|reference]`` (N > 1 under torchrun).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

TOTAL_ENVS = 65536
T_STEPS = 24
BASELINE_VALUE = None  # no published number exists for this configuration (the reference ships no GPU results)


# Benchmark configurations: (total envs or None, envs per GPU or None, env kwargs, description)
CONFIGS = {
    "0": dict(total=1024, per_gpu=None, env={"obs_dim": 48, "num_actions": 12}, cpu=True,
              desc="single-process CPU PPO fp32: MLPs [512,256,128] ELU, obs 48, 12 actions, 1024 envs"),
    "1": dict(total=65536, per_gpu=None, env={}, desc="PPO MLP actor-critic [512,256,128] ELU, obs 96/99, 29 actions"),
    "2": dict(total=65536, per_gpu=None, env={},
              desc="config 1 + RND [256,256]->16 on critic obs (weight 0.5) + symmetry (2 copies, mirror loss 1.0)"),
    "3": dict(total=None, per_gpu=16384, env={"reset_prob": 0.01},
              desc="recurrent PPO: GRU 256 + MLP head [256,128], obs 96, 29 actions, done p=0.01"),
    "3lstm": dict(total=None, per_gpu=16384, env={"reset_prob": 0.01},
                  desc="recurrent PPO: LSTM 256 + MLP head [256,128], obs 96, 29 actions, done p=0.01"),
    "4a": dict(total=65536, per_gpu=None, env={},
               desc="distillation: teacher [512,256,128] obs 99 -> student [256,256,128] obs 96, MSE, 8 steps/rollout"),
    "4b": dict(total=None, per_gpu=32768, env={},
               desc="PPO heteroscedastic Gaussian, MLPs [1024,1024,512], 262144 envs at 8 GPUs (weak scaling)"),
}


def mirror_maps(seed: int = 7):
    """Seeded signed-permutation mirror: an involution on the 96 state features (pairs swapped, signs flipped) and
    on the 29 actions; the 3 privileged critic features are symmetric."""
    import torch

    g = torch.Generator().manual_seed(seed)

    def involution(n):
        perm = torch.arange(n)
        order = torch.randperm(n, generator=g)
        for i in range(0, n - 1, 2):
            a, b = int(order[i]), int(order[i + 1])
            perm[a], perm[b] = b, a
        sign = torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0)
        sign = torch.minimum(sign, sign[perm])  # consistent sign on each pair keeps the map an involution
        return perm, sign

    return involution(96), involution(29)


_MIRROR = None


def mirror_obs_actions(env=None, obs=None, actions=None):
    """Symmetry augmentation function of config 2: returns [original; mirrored] observations / actions."""
    import torch

    global _MIRROR
    if _MIRROR is None:
        _MIRROR = mirror_maps()
    (ps, ss), (pa, sa) = _MIRROR
    out_obs = out_act = None
    if obs is not None:
        groups = {}
        for k, v in obs.items():
            m = v.clone()
            m[:, :96] = v[:, ps.to(v.device)] * ss.to(v.device)
            groups[k] = torch.cat([v, m])
        out_obs = type(obs)(groups, batch_size=[2 * obs.batch_size[0]])
    if actions is not None:
        out_act = torch.cat([actions, actions[:, pa.to(actions.device)] * sa.to(actions.device)])
    return out_obs, out_act


def train_cfg(impl: str, config: str = "1") -> dict:
    if config in ("3", "3lstm"):
        return _recurrent_cfg(impl, "gru" if config == "3" else "lstm")
    if config == "4a":
        return _distill_cfg(impl)
    alg = {
        "class_name": "PPO", "num_learning_epochs": 5, "num_mini_batches": 4, "clip_param": 0.2, "gamma": 0.99,
        "lam": 0.95, "value_loss_coef": 1.0, "entropy_coef": 0.01, "learning_rate": 1e-3, "max_grad_norm": 1.0,
        "schedule": "adaptive", "desired_kl": 0.01, "use_clipped_value_loss": True,
    }
    # bf16 GEMMs on both arms: autocast on the reference arm and on any PyTorch-path fallback of this framework
    alg["use_mixed_precision"] = True
    if config == "0":  # CPU, fp32, no observation normalisation, critic on the policy observations
        alg["use_mixed_precision"] = False
        return {
            "num_steps_per_env": T_STEPS, "save_interval": 10**9, "check_for_nan": True,
            "obs_groups": {"actor": ["policy"], "critic": ["policy"]}, "algorithm": alg,
            "actor": {"class_name": "MLPModel", "hidden_dims": [512, 256, 128], "activation": "elu",
                      "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
            "critic": {"class_name": "MLPModel", "hidden_dims": [512, 256, 128], "activation": "elu"},
        }
    return {
        "num_steps_per_env": T_STEPS, "save_interval": 10**9, "check_for_nan": True,
        "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "algorithm": alg,
        "actor": {"class_name": "MLPModel", "hidden_dims": [512, 256, 128], "activation": "elu",
                  "obs_normalization": True,
                  "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": [512, 256, 128], "activation": "elu",
                   "obs_normalization": True},
    } if config != "4b" else _hetero_wide_cfg(alg)


def _apply_config_2(cfg: dict) -> dict:
    cfg["algorithm"]["rnd_cfg"] = {"num_outputs": 16, "predictor_hidden_dims": [256, 256],
                                   "target_hidden_dims": [256, 256], "weight": 0.5}
    cfg["algorithm"]["symmetry_cfg"] = {"data_augmentation_func": mirror_obs_actions, "use_data_augmentation": True,
                                        "use_mirror_loss": True, "mirror_loss_coeff": 1.0}
    cfg["obs_groups"]["rnd_state"] = ["critic"]
    return cfg


def _hetero_wide_cfg(alg: dict) -> dict:
    return {
        "num_steps_per_env": T_STEPS, "save_interval": 10**9, "check_for_nan": True,
        "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "algorithm": alg,
        "actor": {"class_name": "MLPModel", "hidden_dims": [1024, 1024, 512], "activation": "elu",
                  "obs_normalization": True,
                  "distribution_cfg": {"class_name": "HeteroscedasticGaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": [1024, 1024, 512], "activation": "elu",
                   "obs_normalization": True},
    }


def _recurrent_cfg(impl: str, rnn_type: str) -> dict:
    alg = {"class_name": "PPO", "num_learning_epochs": 5, "num_mini_batches": 4, "learning_rate": 1e-3,
           "schedule": "adaptive", "desired_kl": 0.01, "max_grad_norm": 1.0, "use_mixed_precision": True}
    model = {"class_name": "RNNModel", "hidden_dims": [256, 128], "activation": "elu", "obs_normalization": True,
             "rnn_type": rnn_type, "rnn_hidden_dim": 256, "rnn_num_layers": 1}
    actor = dict(model, distribution_cfg={"class_name": "GaussianDistribution", "init_std": 1.0})
    return {"num_steps_per_env": T_STEPS, "save_interval": 10**9, "check_for_nan": True,
            "obs_groups": {"actor": ["policy"], "critic": ["policy"]}, "algorithm": alg, "actor": actor,
            "critic": dict(model)}


def _distill_cfg(impl: str) -> dict:
    alg = {"class_name": "Distillation", "num_learning_epochs": 1, "gradient_length": 3, "learning_rate": 1e-3,
           "max_grad_norm": 1.0, "loss_type": "mse", "use_mixed_precision": True}
    return {"num_steps_per_env": T_STEPS, "save_interval": 10**9, "check_for_nan": True,
            "obs_groups": {"student": ["policy"], "teacher": ["critic"]}, "algorithm": alg,
            "student": {"class_name": "MLPModel", "hidden_dims": [256, 256, 128], "activation": "elu",
                        "obs_normalization": True,
                        "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
            "teacher": {"class_name": "MLPModel", "hidden_dims": [512, 256, 128], "activation": "elu",
                        "obs_normalization": True}}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons every 200 ms while active."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]) -> None:
        self.gpus = gpus
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                      "-i", ",".join(map(str, self.gpus))], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.rows.append([x.strip() for x in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 9:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_info() -> tuple[int, int, int]:
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK",
                                                                                                      "0"))


ENV_STEP = "PyTorch ops (cuBLAS matmuls + elementwise), the same step code on both arms"


def make_env(num_envs: int, device: str, host_noise: bool, seed: int, inplace_obs: bool = False, **env_kw):
    """The benchmark environment: the PyTorch-op step of the synthetic environment on both arms (none of this
    framework's kernels run inside it). ``inplace_obs`` rewrites the observations in place instead of alternating two
    buffers (same device work); this framework's engines copy observations when they act, which lets its runner
    capture the whole rollout, environment step included, as one CUDA graph. The unmodified reference keeps a
    reference to the observations it acted on, so its arm gets the alternating buffers. Host noise copies are
    double-buffered on a copy stream on both arms."""
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv, humanoid_like

    if "obs_dim" in env_kw:  # config 0: the plain linear-Gaussian environment
        return LinearGaussianVecEnv(num_envs, device=device, seed=seed, fused=False, **env_kw)
    return humanoid_like(num_envs, device=device, seed=seed, host_noise=host_noise, fused=False,
                         inplace_obs=inplace_obs, rollout_steps=T_STEPS if host_noise else None, **env_kw)


def timed_learn_cpu(runner, steps: int, warmup: int) -> float:
    """Seconds per iteration on the host clock (CPU configuration)."""
    runner.learn(warmup)
    t0 = time.perf_counter()
    runner.learn(steps)
    return (time.perf_counter() - t0) / steps


def timed_learn(runner, steps: int, warmup: int, world: int, counter=None) -> float:
    """Seconds per iteration (device time), max over ranks. The first warm-up iteration runs eagerly (CUDA graphs are
    captured from the second one on); with ``counter`` this framework's kernel launches of that iteration are counted,
    which equals the launches of every later (replayed) iteration."""
    import torch

    if counter is not None and warmup > 0:
        with counter:
            runner.learn(1)
        warmup -= 1
    runner.learn(warmup)
    timer = getattr(runner, "section_timer", None)
    if timer is not None:
        timer.totals.clear()  # section times of the timed iterations only (capture iterations bracket host time)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    runner.learn(steps)
    stop.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = start.elapsed_time(stop) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms / 1000.0


def build_runner(impl: str, env, device: str, config: str = "1", sections: bool = False, b200: dict | None = None):
    cfg = train_cfg(impl, config)
    if config == "2":
        cfg = _apply_config_2(cfg)
    if impl == "ours" and b200:
        cfg["algorithm"].setdefault("b200_cfg", {}).update(b200)
    if sections and impl == "ours":
        cfg["algorithm"].setdefault("b200_cfg", {})["section_timing"] = True
    distill = config == "4a"
    if impl == "reference":
        if distill:
            from rsl_rl.runners import DistillationRunner as RefRunner  # noqa: the unmodified reference
        else:
            from rsl_rl.runners import OnPolicyRunner as RefRunner  # noqa: the unmodified reference
        runner = RefRunner(env, cfg, log_dir=None, device=device)
    else:
        if distill:
            from tt_rsl_rl_b200.runners import DistillationRunner as Runner
        else:
            from tt_rsl_rl_b200.runners import OnPolicyRunner as Runner
        runner = Runner(env, cfg, log_dir=None, device=device)
    if distill:
        runner.alg.teacher_loaded = True  # random-init frozen teacher (no checkpoint is available offline)
    return runner


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--total-envs", type=int, default=None,
                    help="environments over all ranks (default: the configuration's; smaller for profiling)")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="1", help="benchmark configuration")
    ap.add_argument("--b200-cfg", default=None,
                    help="JSON object of backend options for this framework's arm (b200_cfg), e.g. '{\"model_streams\": 1}'")
    ap.add_argument("--sections", action="store_true",
                    help="also report rollout / returns / update device milliseconds (CUDA events; ours only)")
    args = ap.parse_args()
    conf = CONFIGS[args.config]
    world, rank, local_rank = dist_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")

    if args.impl == "reference":
        import baseline

        if not baseline.reference_available():
            print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}))
            return
        baseline.add_reference_to_path()

    import torch

    if conf.get("cpu"):
        run_cpu(args, conf)
        return
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    torch.cuda.set_device(local_rank)
    device = f"cuda:{local_rank}"
    # the unmodified reference's runner initialises the process group itself (rsl_rl/runners/on_policy_runner.py
    # _configure_multi_gpu) and refuses an existing one; this framework's runner accepts either
    if world > 1 and not torch.distributed.is_initialized() and args.impl != "reference":
        import datetime

        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device(device),
                                             timeout=datetime.timedelta(seconds=120))
    torch.manual_seed(1 + rank)
    if args.total_envs is not None:
        total_envs = args.total_envs
    elif conf["total"] is not None:
        total_envs = conf["total"]
    else:
        total_envs = conf["per_gpu"] * world
    n_local = total_envs // world
    env_kw = conf["env"]

    inplace_obs = args.impl == "ours"
    # The reference arm measures both numbers with one runner (the unmodified reference's runner initialises the
    # process group itself and refuses a second initialisation): its environment owns the pinned noise pool from the
    # start and switches from device noise to host noise between the two measurements. This framework's arm captures
    # its rollout in a graph, so its end-to-end measurement gets a runner of its own.
    one_runner = args.impl == "reference" and not args.no_e2e
    env = make_env(n_local, device, host_noise=one_runner, seed=rank, inplace_obs=inplace_obs, **env_kw)
    if one_runner:
        env.host_noise = False
    b200 = json.loads(args.b200_cfg) if args.b200_cfg else None
    runner = build_runner(args.impl, env, device, args.config, sections=args.sections, b200=b200)
    sampler = ClockSampler([local_rank]) if local_rank == 0 else None
    if sampler:
        sampler.__enter__()
    counter = None
    host_reads = None
    if args.impl == "ours":
        from tt_rsl_rl_b200.ops import count_launches
        from tt_rsl_rl_b200.utils.timer import HostTransfers

        counter = count_launches()
        HostTransfers.reset()
    s_per_iter = timed_learn(runner, args.steps, args.warmup, world, counter)
    if args.impl == "ours":
        snap = HostTransfers.snapshot()  # over warm-up + timed iterations
        host_reads = {"calls_per_step": snap["calls"] / (args.steps + args.warmup),
                      "bytes_per_step": snap["bytes"] / (args.steps + args.warmup)}
    if sampler:
        sampler.__exit__()
    samples = total_envs * T_STEPS
    value = samples / s_per_iter

    e2e = None
    if not args.no_e2e:
        if one_runner:
            env.host_noise = True
            runner2 = runner
        else:
            env2 = make_env(n_local, device, host_noise=True, seed=rank, inplace_obs=inplace_obs, **env_kw)
            runner2 = build_runner(args.impl, env2, device, args.config, b200=b200)
        e2e_s = timed_learn(runner2, args.steps, args.warmup, world)
        h2d = T_STEPS * n_local * 96 * 4
        e2e = {"value": samples / e2e_s, "unit": "samples/s", "ms_per_step": e2e_s * 1e3,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 20 if args.impl == "ours" else 16,
               "input": "environment process noise copied from pinned host memory every env step"}

    launches = counter.n if counter is not None else None
    sections = None
    timer = getattr(runner, "section_timer", None)
    if args.sections and timer is not None and timer.enabled:
        sections = {k: v / args.steps for k, v in timer.totals.items()}  # ms per timed iteration

    if rank == 0:
        line = {
            "metric": "PPO train samples/s (box, max over ranks)",
            "value": value,
            "unit": "samples/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": s_per_iter * 1e3,
            "s_per_iter": s_per_iter,
            "higher_is_better": True,
            "scaling": "strong" if conf["total"] is not None and args.total_envs is None else "weak",
            "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
            "dtype": "bf16",
            "data": "synthetic (seeded linear-Gaussian env), random-init weights",
            "config": {"model": conf["desc"], "baseline_config": args.config,
                       "global_batch": samples, "seq_len": T_STEPS, "num_envs_total": total_envs,
                       "epochs": 5, "minibatches": 4, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2 (rollout arena >> 126 MB)",
                       "env_step": ENV_STEP},
            "e2e": e2e,
            "gpu_launches": launches,
            "engine_host_reads": host_reads,
            "sections_ms": sections,
            "clocks": sampler.summary() if sampler else None,
        }
        if args.impl == "reference":
            line["impl"] = "reference"
        print(json.dumps(line))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_cpu(args, conf) -> None:
    """Config 0: one process on the host CPU, fp32, timed with the host clock."""
    import torch

    if args.gpus != 1:
        raise SystemExit("config 0 is a single-process CPU configuration")
    torch.manual_seed(1)
    env = make_env(conf["total"], "cpu", host_noise=False, seed=0, **conf["env"])
    runner = build_runner(args.impl, env, "cpu", args.config)
    s_per_iter = timed_learn_cpu(runner, args.steps, args.warmup)
    samples = conf["total"] * T_STEPS
    line = {
        "metric": "PPO train samples/s (box, max over ranks)", "value": samples / s_per_iter, "unit": "samples/s",
        "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "ms_per_step": s_per_iter * 1e3,
        "s_per_iter": s_per_iter, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic (seeded linear-Gaussian env), random-init weights",
        "config": {"model": conf["desc"], "baseline_config": "0", "global_batch": samples, "seq_len": T_STEPS,
                   "num_envs_total": conf["total"], "epochs": 5, "minibatches": 4, "parallelism": "cpu",
                   "timing": "host clock (no device)", "threads": torch.get_num_threads()},
        "e2e": None, "gpu_launches": 0, "clocks": None,
    }
    if args.impl == "reference":
        line["impl"] = "reference"
    print(json.dumps(line))


if __name__ == "__main__":
    main()
