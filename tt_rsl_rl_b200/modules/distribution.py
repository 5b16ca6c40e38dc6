"""Output distributions of stochastic models.

The public interface is rsl_rl's (``rsl_rl/modules/distribution.py``): the class names, the constructor arguments,
the parameter names ``std_param`` / ``log_std_param`` (checkpoint keys), the MLP head layouts (``A`` outputs, or
``[..., 2, A]`` for the two-slice heads) and the methods the models and algorithms call.

Design of this package:

* :class:`DiagonalNormal` writes out the closed forms of a diagonal Gaussian (density, entropy, KL divergence and
  sampling) once, for both Gaussian heads. They are the formulas the fused CUDA kernels evaluate (rollout sampling,
  PPO loss and its gradients); here they are spelled in the operation order of ``torch.distributions.Normal``, which
  rsl_rl uses, so that values, gradients and random draws agree with it bit for bit.
* :class:`StdTransform` is the map from a raw value to a standard deviation: clamped directly (``"scalar"``) or
  clamped in log space and exponentiated (``"log"``). The state-independent head applies it to its parameter, the
  state-dependent (heteroscedastic) head to the second output slice.
* The Beta head rescales ``torch.distributions.Beta`` to an action interval.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
from torch.distributions import Beta

# constants of the Gaussian density and entropy, as Python floats in the form torch's Normal evaluates them
_LOG_NORM = math.log(math.sqrt(2 * math.pi))
_ENTROPY_OFFSET = 0.5 + 0.5 * math.log(2 * math.pi)
_MIN_STD = 1e-6


class DiagonalNormal:
    """A batch of independent normals ``N(loc, scale^2)``; ``loc`` and ``scale`` are broadcast to one shape."""

    __slots__ = ("loc", "scale")

    def __init__(self, loc: torch.Tensor, scale: torch.Tensor) -> None:
        self.loc, self.scale = torch.broadcast_tensors(loc, scale)

    def sample(self) -> torch.Tensor:
        with torch.no_grad():
            return torch.normal(self.loc, self.scale)

    def log_density(self, x: torch.Tensor) -> torch.Tensor:
        """Element-wise ``log N(x; loc, scale^2)``."""
        var = self.scale**2
        return -((x - self.loc) ** 2) / (2 * var) - self.scale.log() - _LOG_NORM

    def entropy(self) -> torch.Tensor:
        return _ENTROPY_OFFSET + torch.log(self.scale)

    @staticmethod
    def kl(p_loc, p_scale, q_loc, q_scale) -> torch.Tensor:
        """Element-wise ``KL(N(p) || N(q))``."""
        var_ratio = (p_scale / q_scale).pow(2)
        t1 = ((p_loc - q_loc) / q_scale).pow(2)
        return 0.5 * (var_ratio + t1 - 1 - var_ratio.log())


class StdTransform:
    """Raw value -> standard deviation, for ``kind`` ``"scalar"`` (clamp) or ``"log"`` (clamp the log, exp).

    The range is given in std space for both kinds; its lower end is raised to at least 1e-6.
    """

    def __init__(self, kind: str, std_range: tuple[float, float]) -> None:
        if kind not in ("scalar", "log"):
            raise ValueError(f"std_type must be 'scalar' or 'log', got {kind!r}")
        self.kind = kind
        lo, hi = max(float(std_range[0]), _MIN_STD), float(std_range[1])
        self.std_range = [lo, hi]
        self.log_std_range = [math.log(lo), math.log(hi)]

    @property
    def param_name(self) -> str:
        return "std_param" if self.kind == "scalar" else "log_std_param"

    def __call__(self, raw: torch.Tensor) -> torch.Tensor:
        if self.kind == "scalar":
            return raw.clamp(self.std_range[0], self.std_range[1])
        return torch.exp(raw.clamp(self.log_std_range[0], self.log_std_range[1]))

    def initial_param(self, std: float, n: int) -> torch.Tensor:
        """A state-independent parameter vector that yields ``std`` everywhere."""
        ones = std * torch.ones(n)
        return ones if self.kind == "scalar" else torch.log(ones)

    def initial_bias(self, std: float) -> float:
        """Bias of a predicted-std output unit that yields ``std`` for a zero weight row."""
        return std if self.kind == "scalar" else float(torch.log(torch.tensor(std + 1e-7)))


class Distribution(nn.Module):
    """Interface of an output distribution driven by an MLP output (rsl_rl's abstract base)."""

    def __init__(self, output_dim: int) -> None:
        super().__init__()
        self.output_dim = output_dim

    def update(self, mlp_output: torch.Tensor) -> None:
        """Set the distribution from a raw MLP output."""
        raise NotImplementedError

    def sample(self) -> torch.Tensor:
        raise NotImplementedError

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        """The mode / mean extracted from a raw MLP output."""
        raise NotImplementedError

    def as_deterministic_output_module(self) -> nn.Module:
        """Export-friendly module computing :meth:`deterministic_output`."""
        raise NotImplementedError

    @property
    def input_dim(self) -> int | list[int]:
        """Output shape the MLP must produce for this distribution."""
        raise NotImplementedError

    @property
    def mean(self) -> torch.Tensor:
        raise NotImplementedError

    @property
    def std(self) -> torch.Tensor:
        raise NotImplementedError

    @property
    def entropy(self) -> torch.Tensor:
        """Entropy summed over the last dimension."""
        raise NotImplementedError

    @property
    def params(self) -> tuple[torch.Tensor, ...]:
        """Tensors that rebuild the distribution (stored in the rollout, used by :meth:`kl_divergence`)."""
        raise NotImplementedError

    def log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        """Log-probability summed over the last dimension."""
        raise NotImplementedError

    def kl_divergence(self, old_params: tuple[torch.Tensor, ...], new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        """``KL(old || new)`` summed over the last dimension."""
        raise NotImplementedError

    def init_mlp_weights(self, mlp: nn.Module) -> None:
        """Distribution-specific initialisation of the MLP's output layer (none by default)."""

    @property
    def ready(self) -> bool:
        """Whether :meth:`update` has been called."""
        return False


def _output_linear(mlp: nn.Module) -> nn.Linear:
    return [m for m in mlp.modules() if isinstance(m, nn.Linear)][-1]


class GaussianDistribution(Distribution):
    """Diagonal Gaussian around the MLP output with a learned (or fixed) state-independent std, clamped to
    ``std_range``; ``std_type`` chooses whether the parameter holds the std or its logarithm."""

    def __init__(self, output_dim: int, init_std: float = 1.0, std_range: tuple[float, float] = (1e-6, 1e6),
                 std_type: str = "scalar", learn_std: bool = True) -> None:
        self._setup(output_dim, std_type, std_range)
        param = nn.Parameter(self._transform.initial_param(init_std, output_dim), requires_grad=learn_std)
        self.register_parameter(self._transform.param_name, param)

    def _setup(self, output_dim: int, std_type: str, std_range) -> None:
        Distribution.__init__(self, output_dim)
        self._transform = StdTransform(std_type, std_range)
        self.std_type = std_type
        self.std_range = self._transform.std_range
        self.log_std_range = self._transform.log_std_range
        self._normal: DiagonalNormal | None = None

    # ---- parameterisation ---------------------------------------------------------------------------------------------
    @property
    def raw_std_param(self) -> nn.Parameter:
        """The learned parameter, ``std_param`` or ``log_std_param``."""
        return getattr(self, self._transform.param_name)

    def current_std(self) -> torch.Tensor:
        """The clamped std vector the parameter stands for."""
        return self._transform(self.raw_std_param)

    def _split(self, mlp_output: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return mlp_output, self.current_std()

    # ---- interface ----------------------------------------------------------------------------------------------------
    def update(self, mlp_output: torch.Tensor) -> None:
        self._normal = DiagonalNormal(*self._split(mlp_output))

    @property
    def ready(self) -> bool:
        return self._normal is not None

    def sample(self) -> torch.Tensor:
        return self._normal.sample()

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output

    def as_deterministic_output_module(self) -> nn.Module:
        return MeanOutput()

    @property
    def input_dim(self) -> int | list[int]:
        return self.output_dim

    @property
    def mean(self) -> torch.Tensor:
        return self._normal.loc

    @property
    def std(self) -> torch.Tensor:
        return self._normal.scale

    @property
    def entropy(self) -> torch.Tensor:
        return self._normal.entropy().sum(dim=-1)

    @property
    def params(self) -> tuple[torch.Tensor, ...]:
        return self._normal.loc, self._normal.scale

    def log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        return self._normal.log_density(outputs).sum(dim=-1)

    def kl_divergence(self, old_params: tuple[torch.Tensor, ...], new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        p = torch.broadcast_tensors(*old_params)
        q = torch.broadcast_tensors(*new_params)
        return DiagonalNormal.kl(p[0], p[1], q[0], q[1]).sum(dim=-1)


class HeteroscedasticGaussianDistribution(GaussianDistribution):
    """Diagonal Gaussian whose std is predicted per state: the MLP outputs ``[..., 2, A]`` = (mean, raw std), the raw
    std mapped by the same clamp (or clamp-in-log + exp) as the parameter head."""

    def __init__(self, output_dim: int, init_std: float = 1.0, std_range: tuple[float, float] = (1e-6, 1e6),
                 std_type: str = "scalar") -> None:
        self._setup(output_dim, std_type, std_range)  # no std parameter: the MLP predicts it
        self.init_std = init_std

    def _split(self, mlp_output: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        loc, raw = torch.unbind(mlp_output, dim=-2)
        return loc, self._transform(raw)

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output[..., 0, :]

    def as_deterministic_output_module(self) -> nn.Module:
        return FirstSliceOutput()

    @property
    def input_dim(self) -> list[int]:
        return [2, self.output_dim]

    def init_mlp_weights(self, mlp: nn.Module) -> None:
        """Zero weight rows and a constant bias for the std outputs: every state starts at ``init_std``."""
        head = _output_linear(mlp)
        nn.init.zeros_(head.weight[self.output_dim :])
        nn.init.constant_(head.bias[self.output_dim :], self._transform.initial_bias(self.init_std))


class BetaDistribution(Distribution):
    """Beta distribution per action, rescaled from ``[0, 1]`` to ``action_range``. The MLP outputs ``[..., 2, A]``
    raw concentrations, each mapped through ``softplus + 1`` (so alpha, beta > 1: unimodal)."""

    def __init__(self, output_dim: int, action_range: tuple[float, float] = (-1.0, 1.0)) -> None:
        super().__init__(output_dim)
        self.action_range = action_range
        self._range_scale = action_range[1] - action_range[0]
        self._range_offset = action_range[0]
        self._log_range_scale = math.log(self._range_scale)
        self._beta_dist: Beta | None = None
        self._alpha: torch.Tensor | None = None
        self._beta: torch.Tensor | None = None
        Beta.set_default_validate_args(False)

    def _to_range(self, unit: torch.Tensor) -> torch.Tensor:
        return unit * self._range_scale + self._range_offset

    def update(self, mlp_output: torch.Tensor) -> None:
        self._alpha, self._beta = _concentrations(mlp_output)
        self._beta_dist = Beta(self._alpha, self._beta)

    @property
    def ready(self) -> bool:
        return self._beta_dist is not None

    def sample(self) -> torch.Tensor:
        return self._to_range(self._beta_dist.sample())

    def deterministic_output(self, mlp_output: torch.Tensor) -> torch.Tensor:
        a, b = _concentrations(mlp_output)
        return self._to_range(a / (a + b))

    def as_deterministic_output_module(self) -> nn.Module:
        return BetaMeanOutput(self._range_scale, self._range_offset)

    @property
    def input_dim(self) -> list[int]:
        return [2, self.output_dim]

    @property
    def mean(self) -> torch.Tensor:
        return self._to_range(self._alpha / (self._alpha + self._beta))

    @property
    def std(self) -> torch.Tensor:
        return self._beta_dist.stddev * self._range_scale

    @property
    def entropy(self) -> torch.Tensor:
        return self._beta_dist.entropy().sum(dim=-1)

    @property
    def params(self) -> tuple[torch.Tensor, ...]:
        return self._alpha, self._beta

    def log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        """Density of the rescaled variable: the unit-interval density minus log(scale), the unit value kept
        1e-6 inside the interval."""
        unit = ((outputs - self._range_offset) / self._range_scale).clamp(1e-6, 1.0 - 1e-6)
        return (self._beta_dist.log_prob(unit) - self._log_range_scale).sum(dim=-1)

    def kl_divergence(self, old_params: tuple[torch.Tensor, ...], new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        return torch.distributions.kl_divergence(Beta(*old_params), Beta(*new_params)).sum(dim=-1)

    def init_mlp_weights(self, mlp: nn.Module) -> None:
        """The beta concentrations start equal to the alpha ones' offset (zero rows and bias)."""
        head = _output_linear(mlp)
        nn.init.zeros_(head.weight[self.output_dim :])
        nn.init.zeros_(head.bias[self.output_dim :])


def _concentrations(mlp_output: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    a_raw, b_raw = torch.unbind(mlp_output, dim=-2)
    return nn.functional.softplus(a_raw) + 1.0, nn.functional.softplus(b_raw) + 1.0


# ---- export modules (TorchScript / ONNX): raw MLP output -> deterministic action ------------------------------------
class MeanOutput(nn.Module):
    def forward(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output


class FirstSliceOutput(nn.Module):
    def forward(self, mlp_output: torch.Tensor) -> torch.Tensor:
        return mlp_output[..., 0, :]


class BetaMeanOutput(nn.Module):
    def __init__(self, range_scale: float, range_offset: float) -> None:
        super().__init__()
        self.range_scale = range_scale
        self.range_offset = range_offset

    def forward(self, mlp_output: torch.Tensor) -> torch.Tensor:
        a_raw, b_raw = torch.unbind(mlp_output, dim=-2)
        a = nn.functional.softplus(a_raw) + 1.0
        b = nn.functional.softplus(b_raw) + 1.0
        return a / (a + b) * self.range_scale + self.range_offset
