"""An environment that does no work, for measuring the algorithm alone.

Observations are drawn once (seeded) and returned unchanged by every step, with constant small rewards, no dones and no
time-outs; ``step`` costs nothing beyond returning references. The reference plugin's algorithm-cost benchmark uses an
environment with the same role (``scripts/bench_matrix.py:34-51``).
"""

from __future__ import annotations

import torch

from ..utils.tensordict import TensorDict
from .vec_env import VecEnv


class NullVecEnv(VecEnv):
    def __init__(self, num_envs: int, groups: dict[str, int] | None = None, num_actions: int = 29, seed: int = 0,
                 device: str | torch.device = "cpu", max_episode_length: int = 1000) -> None:
        groups = groups or {"policy": 96, "critic": 99}
        self.num_envs = num_envs
        self.num_actions = num_actions
        self.device = torch.device(device)
        self.max_episode_length = max_episode_length
        self.step_dt = 0.02
        self.cfg = {"env": "NullVecEnv", "num_envs": num_envs, "groups": dict(groups), "num_actions": num_actions}
        gen = torch.Generator().manual_seed(seed)
        self.episode_length_buf = torch.zeros(num_envs, dtype=torch.long, device=self.device)
        self._obs = TensorDict({g: torch.randn(num_envs, d, generator=gen).to(self.device) for g, d in groups.items()},
                               batch_size=[num_envs], device=self.device)
        self._rewards = (0.1 * torch.randn(num_envs, generator=gen)).to(self.device)
        self._dones = torch.zeros(num_envs, device=self.device)
        self._extras = {"time_outs": torch.zeros(num_envs, device=self.device)}

    @property
    def unwrapped(self):
        return self

    def get_observations(self):
        return self._obs

    def step(self, actions: torch.Tensor):
        return self._obs, self._rewards, self._dones, dict(self._extras)


__all__ = ["NullVecEnv"]
