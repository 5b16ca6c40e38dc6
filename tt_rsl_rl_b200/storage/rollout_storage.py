"""Rollout buffers ``[T, N, ...]`` and minibatch generators (``rsl_rl/storage/rollout_storage.py``).

This is the PyTorch storage used by the CPU path and by recurrent / distillation training. The fused CUDA PPO path
keeps its rollout in the engine's preallocated device arena (``tt_rsl_rl_b200/engine/buffers.py``) and produces the
same minibatches with the gather kernel.
"""

from __future__ import annotations

from collections.abc import Generator

import torch

from ..modules import HiddenState
from ..utils.tensordict import TensorDict
from ..utils.utils import split_and_pad_trajectories


class RolloutStorage:
    class Transition:
        """One environment step's worth of data, filled incrementally during the rollout."""

        def __init__(self) -> None:
            self.observations = None
            self.actions: torch.Tensor | None = None
            self.rewards: torch.Tensor | None = None
            self.dones: torch.Tensor | None = None
            self.values: torch.Tensor | None = None
            self.actions_log_prob: torch.Tensor | None = None
            self.distribution_params: tuple[torch.Tensor, ...] | None = None
            self.privileged_actions: torch.Tensor | None = None
            self.hidden_states: tuple[HiddenState, HiddenState] = (None, None)

        def clear(self) -> None:
            self.__init__()

    class Batch:
        """A minibatch yielded by the generators; unused fields stay ``None``."""

        def __init__(self, observations=None, actions=None, values=None, advantages=None, returns=None,
                     old_actions_log_prob=None, old_distribution_params=None,
                     hidden_states: tuple[HiddenState, HiddenState] = (None, None), masks=None,
                     privileged_actions=None, dones=None) -> None:
            self.observations = observations
            self.actions = actions
            self.values = values
            self.advantages = advantages
            self.returns = returns
            self.old_actions_log_prob = old_actions_log_prob
            self.old_distribution_params = old_distribution_params
            self.privileged_actions = privileged_actions
            self.dones = dones
            self.hidden_states = hidden_states
            self.masks = masks

    def __init__(self, training_type: str, num_envs: int, num_transitions_per_env: int, obs,
                 actions_shape: tuple[int, ...] | list[int], device: str = "cpu") -> None:
        self.training_type = training_type
        self.device = device
        self.num_transitions_per_env = T = num_transitions_per_env
        self.num_envs = N = num_envs
        self.actions_shape = actions_shape
        self.observations = TensorDict(
            {k: torch.zeros(T, *v.shape, dtype=v.dtype, device=device) for k, v in obs.items()},
            batch_size=[T, N], device=device,
        )
        self.rewards = torch.zeros(T, N, 1, device=device)
        self.actions = torch.zeros(T, N, *actions_shape, device=device)
        self.dones = torch.zeros(T, N, 1, device=device).byte()
        if training_type == "distillation":
            self.privileged_actions = torch.zeros(T, N, *actions_shape, device=device)
        if training_type == "rl":
            self.values = torch.zeros(T, N, 1, device=device)
            self.actions_log_prob = torch.zeros(T, N, 1, device=device)
            self.distribution_params: tuple[torch.Tensor, ...] | None = None
            self.returns = torch.zeros(T, N, 1, device=device)
            self.advantages = torch.zeros(T, N, 1, device=device)
        self.saved_hidden_state_a: list[torch.Tensor] | None = None
        self.saved_hidden_state_c: list[torch.Tensor] | None = None
        self.step = 0

    def add_transition(self, transition: Transition) -> None:
        if self.step >= self.num_transitions_per_env:
            raise OverflowError("Rollout buffer overflow! You should call clear() before adding new transitions.")
        t = self.step
        self.observations[t].copy_(transition.observations)
        self.actions[t].copy_(transition.actions)
        self.rewards[t].copy_(transition.rewards.view(-1, 1))
        self.dones[t].copy_(transition.dones.view(-1, 1))
        if self.training_type == "distillation":
            self.privileged_actions[t].copy_(transition.privileged_actions)
        if self.training_type == "rl":
            self.values[t].copy_(transition.values)
            self.actions_log_prob[t].copy_(transition.actions_log_prob.view(-1, 1))
            if self.distribution_params is None:
                self.distribution_params = tuple(
                    torch.zeros(self.num_transitions_per_env, *p.shape, device=self.device)
                    for p in transition.distribution_params
                )
            for buf, p in zip(self.distribution_params, transition.distribution_params):
                buf[t].copy_(p)
        self._save_hidden_states(transition.hidden_states)
        self.step += 1

    def clear(self) -> None:
        self.step = 0

    # ---- generators ---------------------------------------------------------------------------------------------------
    def generator(self) -> Generator[Batch, None, None]:
        """Distillation: one batch per time step, in order."""
        if self.training_type != "distillation":
            raise ValueError("This function is only available for distillation training.")
        for t in range(self.num_transitions_per_env):
            yield RolloutStorage.Batch(observations=self.observations[t], privileged_actions=self.privileged_actions[t],
                                       dones=self.dones[t])

    def mini_batch_generator(self, num_mini_batches: int, num_epochs: int = 8,
                             indices: torch.Tensor | None = None) -> Generator[Batch, None, None]:
        """Shuffled flat minibatches; one permutation per call, reused by every epoch.

        ``indices`` (optional) injects the permutation, which lets tests drive this generator and the CUDA gather
        kernel with the same sample order.
        """
        if self.training_type != "rl":
            raise ValueError("This function is only available for reinforcement learning training.")
        total = self.num_envs * self.num_transitions_per_env
        if not 1 <= num_mini_batches <= total:
            raise ValueError("num_mini_batches must be between 1 and the rollout batch size.")
        if indices is None:
            indices = torch.randperm(total, requires_grad=False, device=self.device)
        obs = self.observations.flatten(0, 1)
        actions = self.actions.flatten(0, 1)
        values = self.values.flatten(0, 1)
        returns = self.returns.flatten(0, 1)
        logp = self.actions_log_prob.flatten(0, 1)
        adv = self.advantages.flatten(0, 1)
        params = tuple(p.flatten(0, 1) for p in self.distribution_params)
        for _ in range(num_epochs):
            for i in range(num_mini_batches):
                idx = indices[i * total // num_mini_batches : (i + 1) * total // num_mini_batches]
                yield RolloutStorage.Batch(
                    observations=obs[idx], actions=actions[idx], values=values[idx], advantages=adv[idx],
                    returns=returns[idx], old_actions_log_prob=logp[idx],
                    old_distribution_params=tuple(p[idx] for p in params),
                )

    def recurrent_mini_batch_generator(self, num_mini_batches: int,
                                       num_epochs: int = 8) -> Generator[Batch, None, None]:
        """Minibatches of whole environments; observations split into zero-padded trajectories at dones."""
        if self.training_type != "rl":
            raise ValueError("This function is only available for reinforcement learning training.")
        if not 1 <= num_mini_batches <= self.num_envs:
            raise ValueError("num_mini_batches must be between 1 and the number of environments.")
        padded_obs, traj_masks = split_and_pad_trajectories(self.observations, self.dones)
        dones = self.dones.squeeze(-1)
        starts = torch.zeros_like(dones, dtype=torch.bool)
        starts[1:] = dones[:-1]
        starts[0] = True
        starts_env_major = starts.permute(1, 0)
        N = self.num_envs
        for _ in range(num_epochs):
            first = 0
            for i in range(num_mini_batches):
                lo = i * N // num_mini_batches
                hi = (i + 1) * N // num_mini_batches
                last = first + int(torch.sum(starts[:, lo:hi]))
                h_a = self._trajectory_hidden(self.saved_hidden_state_a, starts_env_major, first, last)
                h_c = self._trajectory_hidden(self.saved_hidden_state_c, starts_env_major, first, last)
                yield RolloutStorage.Batch(
                    observations=padded_obs[:, first:last], actions=self.actions[:, lo:hi],
                    values=self.values[:, lo:hi], advantages=self.advantages[:, lo:hi],
                    returns=self.returns[:, lo:hi], old_actions_log_prob=self.actions_log_prob[:, lo:hi],
                    old_distribution_params=tuple(p[:, lo:hi] for p in self.distribution_params),
                    hidden_states=(h_a, h_c), masks=traj_masks[:, first:last],
                )
                first = last

    @staticmethod
    def _trajectory_hidden(saved: list[torch.Tensor] | None, starts_env_major: torch.Tensor, first: int, last: int):
        """Hidden states at trajectory starts, ``[layers, num_traj, H]`` (a tuple for LSTMs)."""
        if saved is None:
            return None
        # saved: [T, layers, N, H] -> [N, T, layers, H], select trajectory starts (env-major) -> [num_traj, layers, H]
        states = [s.permute(2, 0, 1, 3)[starts_env_major][first:last].transpose(1, 0).contiguous() for s in saved]
        return states[0] if len(states) == 1 else tuple(states)

    def _save_hidden_states(self, hidden_states: tuple[HiddenState, HiddenState]) -> None:
        if hidden_states == (None, None):
            return
        for which, hs in (("a", hidden_states[0]), ("c", hidden_states[1])):
            if hs is None:
                continue
            parts = hs if isinstance(hs, tuple) else (hs,)
            attr = f"saved_hidden_state_{which}"
            if getattr(self, attr) is None:
                setattr(self, attr, [torch.zeros(self.observations.shape[0], *p.shape, device=self.device)
                                     for p in parts])
            for buf, p in zip(getattr(self, attr), parts):
                buf[self.step].copy_(p)
