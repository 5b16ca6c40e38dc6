"""Random Network Distillation (``rsl_rl/extensions/rnd.py``): intrinsic reward = distance between a frozen random
target MLP and a trained predictor MLP on the ``rnd_state`` observation set.

State-dict layout (``predictor``, ``target``, ``state_normalizer``, ``reward_normalizer``) and the weight schedules
match rsl_rl. The CUDA PPO engine evaluates both MLPs and the distance with the framework's kernels and trains the
predictor in the fused optimizer launch (own Adam, no clipping).
"""

from __future__ import annotations

from typing import Any, NoReturn

import torch
import torch.nn as nn

from ..modules import MLP, EmpiricalDiscountedVariationNormalization, EmpiricalNormalization


class RandomNetworkDistillation(nn.Module):
    def __init__(
        self,
        num_states: int,
        obs_groups: dict,
        num_outputs: int,
        predictor_hidden_dims: tuple[int, ...] | list[int],
        target_hidden_dims: tuple[int, ...] | list[int],
        activation: str = "elu",
        state_normalization: bool = False,
        reward_normalization: bool = False,
        weight: float = 0.0,
        weight_schedule: dict | None = None,
        learning_rate: float = 1e-3,
        device: str = "cpu",
    ) -> None:
        super().__init__()
        self.num_states = num_states
        self.obs_groups = obs_groups
        self.num_outputs = num_outputs
        self.initial_weight = weight
        self.weight = weight
        self.device = device
        self.state_normalization = state_normalization
        self.reward_normalization = reward_normalization
        self.learning_rate = learning_rate
        self.state_normalizer = (EmpiricalNormalization(shape=[num_states], until=int(1.0e8)).to(device)
                                 if state_normalization else nn.Identity())
        self.reward_normalizer = (EmpiricalDiscountedVariationNormalization(shape=[], until=int(1.0e8)).to(device)
                                  if reward_normalization else nn.Identity())
        self.update_counter = 0
        if weight_schedule is not None:
            self.weight_scheduler_params = weight_schedule
            self.weight_scheduler = getattr(self, f"_{weight_schedule['mode']}_weight_schedule")
        else:
            self.weight_scheduler = None
        self.predictor = MLP(num_states, num_outputs, predictor_hidden_dims, activation).to(device)
        self.target = MLP(num_states, num_outputs, target_hidden_dims, activation).to(device)
        self.target.eval()
        self.optimizer = torch.optim.Adam(self.predictor.parameters(), lr=learning_rate)

    def current_weight(self, step: int) -> float:
        """Intrinsic reward weight after ``step`` environment steps (host-side schedule)."""
        if self.weight_scheduler is None:
            return self.initial_weight
        return self.weight_scheduler(step=step, **self.weight_scheduler_params)

    def get_intrinsic_reward(self, obs) -> torch.Tensor:
        self.update_counter += 1
        state = self.state_normalizer(self.get_rnd_state(obs))
        target = self.target(state).detach()
        pred = self.predictor(state).detach()
        reward = torch.linalg.norm(target - pred, dim=1)
        reward = self.reward_normalizer(reward)
        self.weight = self.current_weight(self.update_counter)
        return reward * self.weight

    def compute_loss(self, obs) -> torch.Tensor:
        with torch.no_grad():
            state = self.state_normalizer(self.get_rnd_state(obs))
        return nn.functional.mse_loss(self.predictor(state), self.target(state).detach())

    def forward(self, *args: Any, **kwargs: Any) -> NoReturn:
        raise RuntimeError("Forward method is not implemented. Use get_intrinsic_reward instead.")

    def train(self, mode: bool = True) -> RandomNetworkDistillation:
        self.predictor.train(mode)
        if self.state_normalization:
            self.state_normalizer.train(mode)
        if self.reward_normalization:
            self.reward_normalizer.train(mode)
        return self

    def eval(self) -> RandomNetworkDistillation:
        return self.train(False)

    def get_rnd_state(self, obs) -> torch.Tensor:
        return torch.cat([obs[g] for g in self.obs_groups["rnd_state"]], dim=-1)

    def update_normalization(self, obs) -> None:
        if self.state_normalization:
            self.state_normalizer.update(self.get_rnd_state(obs))

    def _constant_weight_schedule(self, step: int, **kwargs: Any) -> float:
        return self.initial_weight

    def _step_weight_schedule(self, step: int, final_step: int, final_value: float, **kwargs: Any) -> float:
        return self.initial_weight if step < final_step else final_value

    def _linear_weight_schedule(self, step: int, initial_step: int, final_step: int, final_value: float,
                                **kwargs: Any) -> float:
        if step < initial_step:
            return self.initial_weight
        if step > final_step:
            return final_value
        # product before quotient, in upstream's order, so the weight is the same double
        return self.initial_weight + (final_value - self.initial_weight) * (step - initial_step) / (
            final_step - initial_step)


def resolve_rnd_config(alg_cfg: dict, obs, obs_groups: dict[str, list[str]], env) -> dict:
    """Fill ``num_states`` / ``obs_groups`` of ``rnd_cfg`` and scale its weight by ``env.unwrapped.step_dt``."""
    cfg = alg_cfg.get("rnd_cfg")
    if cfg is None:
        alg_cfg["rnd_cfg"] = None
        return alg_cfg
    n = 0
    for g in obs_groups["rnd_state"]:
        if len(obs[g].shape) != 2:
            raise ValueError(f"The RND module only supports 1D observations, got shape {obs[g].shape} for '{g}'.")
        n += obs[g].shape[-1]
    cfg["num_states"] = n
    cfg["obs_groups"] = obs_groups
    cfg["weight"] *= env.unwrapped.step_dt
    return alg_cfg
