"""Shared helpers for the CPU tests: tiny environments and configurations."""

from __future__ import annotations

import copy

import torch

from tt_rsl_rl_b200.env import LinearGaussianVecEnv
from tt_rsl_rl_b200.utils.log_writer import LogWriter


def small_env(num_envs: int = 64, obs_dim: int = 10, num_actions: int = 3, privileged_dim: int = 2, seed: int = 0,
              device: str = "cpu") -> LinearGaussianVecEnv:
    return LinearGaussianVecEnv(num_envs, obs_dim=obs_dim, num_actions=num_actions, privileged_dim=privileged_dim,
                                episode_length=20, reset_prob=0.05, seed=seed, device=device)


def ppo_cfg(hidden=(32, 32), T: int = 8, epochs: int = 2, mbs: int = 2, critic_group: str = "critic", **alg) -> dict:
    a = {"class_name": "PPO", "num_learning_epochs": epochs, "num_mini_batches": mbs, "learning_rate": 1e-3}
    a.update(alg)
    return {
        "num_steps_per_env": T,
        "save_interval": 1000,
        "obs_groups": {"actor": ["policy"], "critic": [critic_group]},
        "algorithm": a,
        "actor": {"class_name": "MLPModel", "hidden_dims": list(hidden), "activation": "elu", "obs_normalization": True,
                  "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": list(hidden), "activation": "elu",
                   "obs_normalization": True},
    }


def copy_cfg(cfg: dict) -> dict:
    return copy.deepcopy(cfg)


def ref_obs(obs, ref_td_cls):
    """Rebuild an observation TensorDict with the reference's TensorDict class."""
    return ref_td_cls({k: v.clone() for k, v in obs.items()}, batch_size=obs.batch_size)


def seed_all(s: int) -> None:
    torch.manual_seed(s)


class RecordingWriter(LogWriter):
    """A LogWriter that records the calls it receives (class-level log, for runner lifecycle tests)."""

    events: list = []

    def __init__(self, log_dir: str, **kwargs) -> None:
        RecordingWriter.events.append(("init", log_dir))

    def add_scalar(self, tag, scalar_value, global_step):
        RecordingWriter.events.append(("scalar", tag, global_step))

    def store_config(self, env_cfg, train_cfg):
        RecordingWriter.events.append(("config",))

    def save_model(self, model_path, it):
        RecordingWriter.events.append(("model", it))

    def save_file(self, path):
        RecordingWriter.events.append(("file", path))

    def save_video(self, video, it):
        RecordingWriter.events.append(("video", str(video), it))

    def stop(self):
        RecordingWriter.events.append(("stop",))

    def abort(self):
        RecordingWriter.events.append(("abort",))
