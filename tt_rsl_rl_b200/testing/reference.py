"""Reference training runs on the seeded test environments: run specifications, configuration builders and helpers
that train with either this framework or the unmodified upstream rsl_rl runner.

The reference plugin has the same roles (``rsl_rl_tt/testing/reference.py:23-248``: run specs per environment, config
builders with RND / symmetry / recurrent variants, teacher checkpoints for distillation, a helper that trains with the
upstream runner). Here one builder serves both implementations:

* ``impl="b200"`` — this framework's runners on ``device`` (``"cpu"``: the PyTorch path; ``"cuda:N"``: the fused
  engines where the configuration allows);
* ``impl="upstream"`` — upstream ``rsl_rl`` (importable as ``rsl_rl``, e.g. an install of the reference) on the CPU,
  the oracle that :mod:`tt_rsl_rl_b200.testing.golden` records curves from.

Both log through :class:`~tt_rsl_rl_b200.utils.log_writer.CsvLogWriter` (``metrics.csv`` in the run's folder).
"""

from __future__ import annotations

import copy
import dataclasses
import importlib
import os
import time
from dataclasses import dataclass

import torch

from ..env.classic import env_class, make_env

CSV_LOGGER = {"class_name": "tt_rsl_rl_b200.utils.log_writer:CsvLogWriter"}
IMPLS = ("b200", "upstream")


@dataclass(frozen=True)
class RunSpec:
    """One reference run: environment count, rollout length, iterations, MLP sizes and the algorithm section.

    ``model`` adds keys to the actor's model config (and to the critic's unless ``critic_model`` is given; ``{}`` keeps
    that model a plain MLP), e.g. ``{"class_name": "RNNModel", "rnn_type": "gru", "rnn_hidden_dim": 64}``."""

    num_envs: int
    num_steps: int
    iterations: int
    hidden: tuple[int, ...]
    algorithm: dict
    init_std: float = 1.0
    obs_normalization: bool = True
    distribution: str = "GaussianDistribution"
    obs_groups: dict | None = None
    model: dict | None = None
    critic_model: dict | None = None


PPO_ALGORITHM = {
    "class_name": "PPO",
    "num_learning_epochs": 5,
    "num_mini_batches": 4,
    "clip_param": 0.2,
    "gamma": 0.99,
    "lam": 0.95,
    "value_loss_coef": 1.0,
    "entropy_coef": 0.005,
    "learning_rate": 1.0e-3,
    "max_grad_norm": 1.0,
    "optimizer": "adam",
    "use_clipped_value_loss": True,
    "schedule": "adaptive",
    "desired_kl": 0.01,
    "normalize_advantage_per_mini_batch": False,
}

SPECS: dict[str, RunSpec] = {
    "cartpole": RunSpec(num_envs=1024, num_steps=24, iterations=100, hidden=(64, 64), algorithm=PPO_ALGORITHM),
    "pendulum": RunSpec(num_envs=1024, num_steps=32, iterations=200, hidden=(64, 64),
                        algorithm={**PPO_ALGORITHM, "gamma": 0.95}),
    # the actions are clipped by the environment, so an entropy bonus would only grow the std
    "tracking12": RunSpec(num_envs=2048, num_steps=24, iterations=300, hidden=(128, 128, 64),
                          algorithm={**PPO_ALGORITHM, "entropy_coef": 0.0}),
    # positions only: a feed-forward policy cannot infer the velocities, a recurrent one can
    "cartpole_po": RunSpec(num_envs=1024, num_steps=24, iterations=150, hidden=(64,), algorithm=PPO_ALGORITHM,
                           model={"class_name": "RNNModel", "rnn_type": "gru", "rnn_hidden_dim": 64,
                                  "rnn_num_layers": 1}),
}

# RND weight per environment; the configuration scales it by the environment's step_dt (upstream rule)
RND_WEIGHT = {"cartpole": 5.0, "cartpole_po": 5.0, "pendulum": 2.0, "tracking12": 5.0}
SYMMETRY_FUNCS = {"cartpole": "cartpole_mirror", "cartpole_po": "cartpole_mirror", "pendulum": "pendulum_mirror",
                  "tracking12": "tracking12_sign_mirror"}


def with_rnd(env_name: str, spec: RunSpec) -> RunSpec:
    """``spec`` with Random Network Distillation on the policy observations (state and reward normalisation on)."""
    rnd = {"predictor_hidden_dims": [64, 64], "target_hidden_dims": [64, 64], "num_outputs": 16, "activation": "elu",
           "state_normalization": True, "reward_normalization": True, "weight": RND_WEIGHT[env_name],
           "learning_rate": 1.0e-3}
    return dataclasses.replace(spec, algorithm={**spec.algorithm, "rnd_cfg": rnd})


def symmetry_cfg(env_name: str, *, data_augmentation: bool = True, mirror_loss: bool = True, coeff: float = 0.2,
                 func: str | None = None) -> dict:
    """``symmetry_cfg`` naming the environment's mirror function in :mod:`tt_rsl_rl_b200.testing.symmetry`."""
    return {"data_augmentation_func": f"tt_rsl_rl_b200.testing.symmetry:{func or SYMMETRY_FUNCS[env_name]}",
            "use_data_augmentation": data_augmentation, "use_mirror_loss": mirror_loss, "mirror_loss_coeff": coeff}


def with_symmetry(env_name: str, spec: RunSpec, **kwargs) -> RunSpec:
    """``spec`` with the symmetry extension (augmentation and mirror loss by default)."""
    return dataclasses.replace(spec, algorithm={**spec.algorithm, "symmetry_cfg": symmetry_cfg(env_name, **kwargs)})


def with_rnn(spec: RunSpec, rnn_type: str = "gru", hidden_dim: int = 64, num_layers: int = 1, actor: bool = True,
             critic: bool = True) -> RunSpec:
    """``spec`` with recurrent models; ``actor`` / ``critic`` False keeps that model a plain MLP."""
    model = {"class_name": "RNNModel", "rnn_type": rnn_type, "rnn_hidden_dim": hidden_dim,
             "rnn_num_layers": num_layers}
    return dataclasses.replace(spec, model=model if actor else {}, critic_model=model if critic else {})


def _dist_cfg(spec: RunSpec) -> dict:
    """``distribution_cfg`` of the spec (Gaussian families take an initial std, the Beta policy has none)."""
    dist = {"class_name": spec.distribution}
    if "Gaussian" in spec.distribution:
        dist["init_std"] = spec.init_std
    return dist


def train_cfg(env_name: str, spec: RunSpec | None = None, logger: dict | None = CSV_LOGGER) -> dict:
    """``OnPolicyRunner`` configuration of ``spec`` (default: the environment's own) on ``env_name``."""
    spec = spec or SPECS[env_name]
    dist = _dist_cfg(spec)
    mlp = {"class_name": "MLPModel", "hidden_dims": list(spec.hidden), "activation": "elu",
           "obs_normalization": spec.obs_normalization}
    critic_extra = (spec.model or {}) if spec.critic_model is None else spec.critic_model
    cfg = {
        "num_steps_per_env": spec.num_steps,
        "save_interval": 10_000,
        "check_for_nan": True,
        "obs_groups": copy.deepcopy(spec.obs_groups or env_class(env_name).obs_groups_cfg),
        "actor": {**mlp, "distribution_cfg": dist, **copy.deepcopy(spec.model or {})},
        "critic": {**mlp, **copy.deepcopy(critic_extra)},
        "algorithm": copy.deepcopy(spec.algorithm),
    }
    if logger is not None:
        cfg["logger"] = dict(logger)
    return cfg


# ---- distillation -----------------------------------------------------------------------------------------------------
# the student sees the policy group; the tracking teacher also sees the privileged group
DISTILL_GROUPS = {
    "cartpole": {"student": ["policy"], "teacher": ["policy"]},
    "pendulum": {"student": ["policy"], "teacher": ["policy"]},
    "tracking12": {"student": ["policy"], "teacher": ["policy", "privileged"]},
}
DISTILL_ITERATIONS = {"cartpole": 60, "pendulum": 100, "tracking12": 100}
DISTILLATION_ALGORITHM = {"class_name": "Distillation", "num_learning_epochs": 2, "gradient_length": 6,
                          "learning_rate": 1.0e-3, "max_grad_norm": 1.0, "loss_type": "mse", "optimizer": "adam"}


def teacher_train_cfg(env_name: str, logger: dict | None = CSV_LOGGER) -> dict:
    """RL configuration whose actor sees the teacher's groups, so its ``actor_state_dict`` loads into the teacher."""
    groups = {"actor": list(DISTILL_GROUPS[env_name]["teacher"]),
              "critic": list(env_class(env_name).obs_groups_cfg["critic"])}
    return train_cfg(env_name, dataclasses.replace(SPECS[env_name], obs_groups=groups), logger)


def distill_cfg(env_name: str, spec: RunSpec | None = None, logger: dict | None = CSV_LOGGER,
                algorithm: dict | None = None, student_model: dict | None = None) -> dict:
    """``DistillationRunner`` configuration: student and teacher MLPs of the spec's size; ``student_model`` adds keys
    to the student's model config (e.g. a recurrent student: ``{"class_name": "RNNModel", "rnn_type": "gru"}``)."""
    spec = spec or SPECS[env_name]
    model = {"class_name": "MLPModel", "hidden_dims": list(spec.hidden), "activation": "elu",
             "obs_normalization": spec.obs_normalization,
             "distribution_cfg": _dist_cfg(spec)}
    cfg = {
        "num_steps_per_env": spec.num_steps,
        "save_interval": 10_000,
        "check_for_nan": True,
        "obs_groups": copy.deepcopy(DISTILL_GROUPS[env_name]),
        "student": {**copy.deepcopy(model), **copy.deepcopy(student_model or {})},
        "teacher": copy.deepcopy(model),
        "algorithm": {**DISTILLATION_ALGORITHM, **(algorithm or {})},
    }
    if logger is not None:
        cfg["logger"] = dict(logger)
    return cfg


# ---- runner construction ----------------------------------------------------------------------------------------------
def upstream_runners():
    """``(OnPolicyRunner, DistillationRunner, TensorDict)`` of upstream rsl_rl.

    Upstream must be importable as ``rsl_rl`` together with a ``tensordict`` package; from a checkout of this
    repository the install under ``baseline/_ref`` (with its ``tensordict`` stand-in) is put on the path."""
    try:
        mod = importlib.import_module("rsl_rl.runners")
        td = importlib.import_module("tensordict")
    except ImportError:
        try:
            baseline = importlib.import_module("baseline")
        except ImportError as exc:
            raise ImportError("upstream rsl_rl is not importable (install it, or run from the repository root so "
                              "baseline/_ref can be found)") from exc
        if not baseline.reference_available():
            raise ImportError("upstream rsl_rl is not installed in baseline/_ref") from None
        baseline.add_reference_to_path()
        mod = importlib.import_module("rsl_rl.runners")
        td = importlib.import_module("tensordict")
    return mod.OnPolicyRunner, mod.DistillationRunner, td.TensorDict


class UpstreamEnvAdapter:
    """Presents a test environment to the upstream runner: observations as upstream's ``TensorDict`` class, every
    other attribute (``episode_length_buf`` included, read and written) forwarded to the wrapped environment."""

    def __init__(self, env, td_cls) -> None:
        object.__setattr__(self, "env", env)
        object.__setattr__(self, "_td_cls", td_cls)

    def __getattr__(self, name):
        return getattr(self.env, name)

    def __setattr__(self, name, value):
        setattr(self.env, name, value)

    @property
    def unwrapped(self):
        return self.env

    def _convert(self, obs):
        return self._td_cls({k: obs[k] for k in obs.keys()}, batch_size=obs.batch_size, device=obs.device)

    def get_observations(self):
        return self._convert(self.env.get_observations())

    def step(self, actions):
        obs, rewards, dones, extras = self.env.step(actions)
        return self._convert(obs), rewards, dones, extras


def _check_impl(impl: str, device: str) -> None:
    if impl not in IMPLS:
        raise ValueError(f"impl must be one of {IMPLS}, got {impl!r}")
    if impl == "upstream" and str(device) != "cpu":
        raise ValueError("the upstream oracle runs on the CPU")


def build_runner(env_name: str, seed: int, log_dir: str | None = None, spec: RunSpec | None = None, *,
                 impl: str = "b200", device: str = "cpu", num_envs: int | None = None,
                 cfg: dict | None = None):
    """Seed torch, build the environment and an ``OnPolicyRunner`` of ``impl``. Returns ``(runner, env, spec)``."""
    _check_impl(impl, device)
    spec = spec or SPECS[env_name]
    torch.manual_seed(seed)
    env = make_env(env_name, num_envs or spec.num_envs, seed=seed, device=device)
    cfg = cfg if cfg is not None else train_cfg(env_name, spec, CSV_LOGGER if log_dir else None)
    if impl == "upstream":
        runner_cls, _, td_cls = upstream_runners()
        return runner_cls(UpstreamEnvAdapter(env, td_cls), cfg, log_dir=log_dir, device="cpu"), env, spec
    from ..runners import OnPolicyRunner

    return OnPolicyRunner(env, cfg, log_dir=log_dir, device=device), env, spec


def _finish_writer(runner) -> None:
    writer = getattr(getattr(runner, "logger", None), "writer", None)
    if writer is not None and hasattr(writer, "stop"):
        writer.stop()  # the last iteration's row is written when the writer stops


def train(env_name: str, seed: int, log_dir: str, *, impl: str = "b200", device: str = "cpu",
          iterations: int | None = None, spec: RunSpec | None = None, num_threads: int | None = None,
          engine: str | None = None, mixed_precision: bool = False) -> dict:
    """Train ``spec`` on ``env_name`` from ``seed``; the metrics land in ``log_dir/metrics.csv``. Returns a summary.

    ``engine`` (this framework only): ``b200_cfg.engine`` of the run, e.g. ``"torch"`` for the PyTorch path on a CUDA
    device; ``mixed_precision``: bf16 autocast on the PyTorch path."""
    if num_threads is not None:
        torch.set_num_threads(num_threads)
    os.makedirs(log_dir, exist_ok=True)
    cfg = None
    if engine is not None or mixed_precision:
        cfg = train_cfg(env_name, spec or SPECS[env_name], CSV_LOGGER if log_dir else None)
        if engine is not None:
            cfg["algorithm"].setdefault("b200_cfg", {})["engine"] = engine
        if mixed_precision:
            cfg["algorithm"]["use_mixed_precision"] = True
    runner, _, spec = build_runner(env_name, seed, log_dir, spec, impl=impl, device=device, cfg=cfg)
    n_it = spec.iterations if iterations is None else iterations
    t0 = time.time()
    runner.learn(num_learning_iterations=n_it, init_at_random_ep_len=True)
    _finish_writer(runner)
    return {"env": env_name, "seed": seed, "impl": impl, "device": str(device), "iterations": n_it,
            "wall_s": time.time() - t0, "num_envs": spec.num_envs, "num_steps": spec.num_steps,
            "num_threads": torch.get_num_threads()}


def make_teacher_checkpoint(env_name: str, path: str, seed: int = 0, iterations: int = 30, num_envs: int = 256,
                            impl: str = "b200") -> str:
    """Train a teacher by PPO on the CPU and save it; its ``actor_state_dict`` loads into a distillation teacher."""
    spec = dataclasses.replace(SPECS[env_name], num_envs=num_envs, iterations=iterations)
    runner, _, _ = build_runner(env_name, seed, None, spec, impl=impl, cfg=teacher_train_cfg(env_name, None))
    runner.learn(num_learning_iterations=iterations, init_at_random_ep_len=True)
    runner.save(path)
    return path


def build_distillation_runner(env_name: str, seed: int, log_dir: str | None, teacher_ckpt: str, *,
                              impl: str = "b200", device: str = "cpu", spec: RunSpec | None = None,
                              num_envs: int | None = None, algorithm: dict | None = None,
                              student_model: dict | None = None):
    """Seed, build the environment and a ``DistillationRunner`` of ``impl``, load the teacher from an RL checkpoint.
    Returns ``(runner, env, spec)``."""
    _check_impl(impl, device)
    spec = spec or SPECS[env_name]
    torch.manual_seed(seed)
    env = make_env(env_name, num_envs or spec.num_envs, seed=seed, device=device)
    cfg = distill_cfg(env_name, spec, CSV_LOGGER if log_dir else None, algorithm, student_model)
    if impl == "upstream":
        _, runner_cls, td_cls = upstream_runners()
        runner = runner_cls(UpstreamEnvAdapter(env, td_cls), cfg, log_dir=log_dir, device="cpu")
    else:
        from ..runners import DistillationRunner

        runner = DistillationRunner(env, cfg, log_dir=log_dir, device=device)
    runner.load(teacher_ckpt, map_location=str(device))  # an RL checkpoint: only the teacher is loaded
    return runner, env, spec


def train_distillation(env_name: str, seed: int, log_dir: str, teacher_ckpt: str, *, impl: str = "b200",
                       device: str = "cpu", iterations: int | None = None, algorithm: dict | None = None,
                       student_model: dict | None = None) -> dict:
    """Distil ``teacher_ckpt`` into a student; metrics in ``log_dir/metrics.csv``. Returns a summary."""
    os.makedirs(log_dir, exist_ok=True)
    runner, _, spec = build_distillation_runner(env_name, seed, log_dir, teacher_ckpt, impl=impl, device=device,
                                                algorithm=algorithm, student_model=student_model)
    n_it = DISTILL_ITERATIONS[env_name] if iterations is None else iterations
    t0 = time.time()
    runner.learn(num_learning_iterations=n_it, init_at_random_ep_len=True)
    _finish_writer(runner)
    return {"env": env_name, "seed": seed, "impl": impl, "device": str(device), "iterations": n_it,
            "wall_s": time.time() - t0, "num_envs": spec.num_envs, "num_steps": spec.num_steps}


__all__ = ["CSV_LOGGER", "DISTILL_GROUPS", "PPO_ALGORITHM", "RunSpec", "SPECS", "UpstreamEnvAdapter",
           "build_distillation_runner", "build_runner", "distill_cfg", "make_teacher_checkpoint", "symmetry_cfg",
           "teacher_train_cfg", "train", "train_cfg", "train_distillation", "upstream_runners", "with_rnd",
           "with_rnn", "with_symmetry"]
