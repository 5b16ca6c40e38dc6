"""Output distributions of stochastic models (``rsl_rl/modules/distribution.py``).

Parameter names (``std_param`` / ``log_std_param``) and MLP head layouts match rsl_rl so checkpoints interoperate.
The fused CUDA path implements the same math in kernels: the Gaussian head (sampling, log-prob) in the rollout kernel
and log-prob/entropy/KL and their gradients in the PPO loss kernel; these classes are the PyTorch definition.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
from torch.distributions import Beta, Normal

LOG_SQRT_2PI = 0.5 * math.log(2.0 * math.pi)


class Distribution(nn.Module):
    """Interface of an output distribution driven by the MLP output."""

    def __init__(self, output_dim: int) -> None:
        super().__init__()
        self.output_dim = output_dim

    def update(self, mlp_output: torch.Tensor) -> None:
        raise NotImplementedError

    def sample(self) -> torch.Tensor:
        raise NotImplementedError

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def as_deterministic_output_module(self) -> nn.Module:
        raise NotImplementedError

    @property
    def input_dim(self) -> int | list[int]:
        raise NotImplementedError

    @property
    def mean(self) -> torch.Tensor:
        raise NotImplementedError

    @property
    def std(self) -> torch.Tensor:
        raise NotImplementedError

    @property
    def entropy(self) -> torch.Tensor:
        raise NotImplementedError

    @property
    def params(self) -> tuple[torch.Tensor, ...]:
        raise NotImplementedError

    def log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def kl_divergence(self, old_params: tuple[torch.Tensor, ...], new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        raise NotImplementedError

    def init_mlp_weights(self, mlp: nn.Module) -> None:
        """Distribution-specific initialisation of the MLP head (default: nothing)."""


def _std_ranges(std_range: tuple[float, float]) -> tuple[list[float], list[float]]:
    lo = max(float(std_range[0]), 1e-6)
    hi = float(std_range[1])
    return [lo, hi], [math.log(lo), math.log(hi)]


class GaussianDistribution(Distribution):
    """Diagonal Gaussian with a state-independent std parameter (``std_type`` "scalar" or "log"), clamped."""

    def __init__(self, output_dim: int, init_std: float = 1.0, std_range: tuple[float, float] = (1e-6, 1e6),
                 std_type: str = "scalar", learn_std: bool = True) -> None:
        super().__init__(output_dim)
        self.std_type = std_type
        if std_type == "scalar":
            self.std_param = nn.Parameter(init_std * torch.ones(output_dim), requires_grad=learn_std)
        elif std_type == "log":
            self.log_std_param = nn.Parameter(torch.log(init_std * torch.ones(output_dim)), requires_grad=learn_std)
        else:
            raise ValueError(f"Unknown standard deviation type: {std_type}. Should be 'scalar' or 'log'.")
        self.std_range, self.log_std_range = _std_ranges(std_range)
        self._distribution: Normal | None = None
        Normal.set_default_validate_args(False)

    def current_std(self) -> torch.Tensor:
        """The clamped std vector implied by the parameter."""
        if self.std_type == "scalar":
            return self.std_param.clamp(self.std_range[0], self.std_range[1])
        return torch.exp(self.log_std_param.clamp(self.log_std_range[0], self.log_std_range[1]))

    def update(self, mlp_output: torch.Tensor) -> None:
        self._distribution = Normal(mlp_output, self.current_std())

    def sample(self) -> torch.Tensor:
        return self._distribution.sample()

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output

    def as_deterministic_output_module(self) -> nn.Module:
        return _IdentityDeterministicOutput()

    @property
    def input_dim(self) -> int:
        return self.output_dim

    @property
    def mean(self) -> torch.Tensor:
        return self._distribution.mean

    @property
    def std(self) -> torch.Tensor:
        return self._distribution.stddev

    @property
    def entropy(self) -> torch.Tensor:
        return self._distribution.entropy().sum(dim=-1)

    @property
    def params(self) -> tuple[torch.Tensor, ...]:
        return (self.mean, self.std)

    def log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        return self._distribution.log_prob(outputs).sum(dim=-1)

    def kl_divergence(self, old_params: tuple[torch.Tensor, ...], new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        return torch.distributions.kl_divergence(Normal(*old_params), Normal(*new_params)).sum(dim=-1)


class HeteroscedasticGaussianDistribution(GaussianDistribution):
    """Diagonal Gaussian whose std is predicted by the MLP: output ``[..., 2, A]`` = (mean, std or log-std)."""

    def __init__(self, output_dim: int, init_std: float = 1.0, std_range: tuple[float, float] = (1e-6, 1e6),
                 std_type: str = "scalar") -> None:
        Distribution.__init__(self, output_dim)
        if std_type not in ("scalar", "log"):
            raise ValueError(f"Unknown standard deviation type: {std_type}. Should be 'scalar' or 'log'.")
        self.std_type = std_type
        self.init_std = init_std
        self.std_range, self.log_std_range = _std_ranges(std_range)
        self._distribution = None
        Normal.set_default_validate_args(False)

    def update(self, mlp_output: torch.Tensor) -> None:
        mean, spread = torch.unbind(mlp_output, dim=-2)
        if self.std_type == "scalar":
            std = spread.clamp(self.std_range[0], self.std_range[1])
        else:
            std = torch.exp(spread.clamp(self.log_std_range[0], self.log_std_range[1]))
        self._distribution = Normal(mean, std)

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output[..., 0, :]

    def as_deterministic_output_module(self) -> nn.Module:
        return _FirstSliceDeterministicOutput()

    @property
    def input_dim(self) -> list[int]:
        return [2, self.output_dim]

    def init_mlp_weights(self, mlp: nn.Module) -> None:
        """Zero the std rows of the last Linear and set their bias to ``init_std`` (or its log)."""
        head = mlp[-2]
        nn.init.zeros_(head.weight[self.output_dim :])
        if self.std_type == "scalar":
            nn.init.constant_(head.bias[self.output_dim :], self.init_std)
        else:
            nn.init.constant_(head.bias[self.output_dim :], float(torch.log(torch.tensor(self.init_std + 1e-7))))


class BetaDistribution(Distribution):
    """Beta distribution on ``[0, 1]`` rescaled to ``action_range``; MLP output ``[..., 2, A]`` through softplus+1."""

    def __init__(self, output_dim: int, action_range: tuple[float, float] = (-1.0, 1.0)) -> None:
        super().__init__(output_dim)
        self.action_range = action_range
        self._range_scale = action_range[1] - action_range[0]
        self._range_offset = action_range[0]
        self._log_range_scale = math.log(self._range_scale)
        self._distribution: Beta | None = None
        self._alpha: torch.Tensor | None = None
        self._beta: torch.Tensor | None = None
        Beta.set_default_validate_args(False)

    @staticmethod
    def _concentrations(mlp_output: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        a_raw, b_raw = torch.unbind(mlp_output, dim=-2)
        return nn.functional.softplus(a_raw) + 1.0, nn.functional.softplus(b_raw) + 1.0

    def update(self, mlp_output: torch.Tensor) -> None:
        self._alpha, self._beta = self._concentrations(mlp_output)
        self._distribution = Beta(self._alpha, self._beta)

    def sample(self) -> torch.Tensor:
        return self._distribution.sample() * self._range_scale + self._range_offset

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        a, b = self._concentrations(mlp_output)
        return a / (a + b) * self._range_scale + self._range_offset

    def as_deterministic_output_module(self) -> nn.Module:
        return _BetaDeterministicOutput(self._range_scale, self._range_offset)

    @property
    def input_dim(self) -> list[int]:
        return [2, self.output_dim]

    @property
    def mean(self) -> torch.Tensor:
        return self._alpha / (self._alpha + self._beta) * self._range_scale + self._range_offset

    @property
    def std(self) -> torch.Tensor:
        return self._distribution.stddev * self._range_scale

    @property
    def entropy(self) -> torch.Tensor:
        return self._distribution.entropy().sum(dim=-1)

    @property
    def params(self) -> tuple[torch.Tensor, ...]:
        return (self._alpha, self._beta)

    def log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        unit = ((outputs - self._range_offset) / self._range_scale).clamp(1e-6, 1.0 - 1e-6)
        return (self._distribution.log_prob(unit) - self._log_range_scale).sum(dim=-1)

    def kl_divergence(self, old_params: tuple[torch.Tensor, ...], new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        return torch.distributions.kl_divergence(Beta(*old_params), Beta(*new_params)).sum(dim=-1)

    def init_mlp_weights(self, mlp: nn.Module) -> None:
        head = mlp[-2]
        nn.init.zeros_(head.weight[self.output_dim :])
        nn.init.zeros_(head.bias[self.output_dim :])


class _IdentityDeterministicOutput(nn.Module):
    def forward(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output


class _FirstSliceDeterministicOutput(nn.Module):
    def forward(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output[..., 0, :]


class _BetaDeterministicOutput(nn.Module):
    def __init__(self, range_scale: float, range_offset: float) -> None:
        super().__init__()
        self.range_scale = range_scale
        self.range_offset = range_offset

    def forward(self, mlp_output: torch.Tensor) -> torch.Tensor:
        a_raw, b_raw = torch.unbind(mlp_output, dim=-2)
        a = nn.functional.softplus(a_raw) + 1.0
        b = nn.functional.softplus(b_raw) + 1.0
        return a / (a + b) * self.range_scale + self.range_offset
