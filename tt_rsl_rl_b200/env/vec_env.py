"""Vectorised environment interface (``rsl_rl/env/vec_env.py``).

An environment exposes ``num_envs``, ``num_actions``, ``max_episode_length``, ``episode_length_buf``, ``device`` and
``cfg``; ``get_observations()`` returns a TensorDict of observation groups and ``step(actions)`` returns
``(obs, rewards [N], dones [N], extras)`` with optional ``extras["time_outs"]`` and ``extras["log"]``.

Optional capability used by the CUDA runner: an environment whose ``step`` performs only asynchronous device work
(no host synchronisation, no allocation after the first call) may set ``graph_capturable = True``; the runner then
captures the whole rollout step (policy inference + environment step + storage) in one CUDA graph.
"""

from __future__ import annotations

from abc import ABC, abstractmethod

import torch


class VecEnv(ABC):
    num_envs: int
    num_actions: int
    max_episode_length: int | torch.Tensor
    episode_length_buf: torch.Tensor
    device: torch.device | str
    cfg: dict | object
    graph_capturable: bool = False

    @abstractmethod
    def get_observations(self):
        """Current observations (a TensorDict of groups). They must stay unchanged until the next step is stored."""
        raise NotImplementedError

    @abstractmethod
    def step(self, actions: torch.Tensor):
        """Apply ``actions [N, num_actions]``; return ``(obs, rewards, dones, extras)``."""
        raise NotImplementedError
