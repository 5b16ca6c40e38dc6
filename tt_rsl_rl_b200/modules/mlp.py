"""Multi-layer perceptron with the parameter names and layout of ``rsl_rl/modules/mlp.py`` (``nn.Sequential`` of
``Linear, act, ..., Linear``), so state dicts are interchangeable with rsl_rl checkpoints."""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..utils.utils import get_param, resolve_nn_activation


class MLP(nn.Sequential):
    """``Linear -> act -> ... -> Linear`` with optional output reshape and last activation.

    A hidden size of ``-1`` means "same as the input size". A tuple ``output_dim`` appends an ``nn.Unflatten`` so the
    output has that trailing shape (used by two-headed distributions).
    """

    __jit_unused_properties__ = ["linears", "activation_name"]

    def __init__(
        self,
        input_dim: int,
        output_dim: int | tuple[int, ...] | list[int],
        hidden_dims: tuple[int, ...] | list[int],
        activation: str = "elu",
        last_activation: str | None = None,
    ) -> None:
        super().__init__()
        act = resolve_nn_activation(activation)
        sizes = [input_dim] + [input_dim if h == -1 else h for h in hidden_dims]
        modules: list[nn.Module] = []
        for fan_in, fan_out in zip(sizes[:-1], sizes[1:]):
            modules += [nn.Linear(fan_in, fan_out), act]
        if isinstance(output_dim, int):
            modules.append(nn.Linear(sizes[-1], output_dim))
        else:
            modules.append(nn.Linear(sizes[-1], math.prod(output_dim)))
            modules.append(nn.Unflatten(dim=-1, unflattened_size=tuple(output_dim)))
        if last_activation is not None:
            modules.append(resolve_nn_activation(last_activation))
        for i, m in enumerate(modules):
            self.add_module(str(i), m)

    @property
    def linears(self) -> list[nn.Linear]:
        """The Linear layers in order."""
        return [m for m in self if isinstance(m, nn.Linear)]

    @property
    def activation_name(self) -> str:
        """Lower-case class name of the hidden activation (e.g. ``"elu"``)."""
        for m in self:
            if not isinstance(m, (nn.Linear, nn.Unflatten)):
                return type(m).__name__.lower()
        return "identity"

    def init_weights(self, scales: float | tuple[float, ...]) -> None:
        """Orthogonal weights with gain ``get_param(scales, module_index)`` and zero biases."""
        for idx, module in enumerate(self):
            if isinstance(module, nn.Linear):
                nn.init.orthogonal_(module.weight, gain=get_param(scales, idx))
                nn.init.zeros_(module.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self:
            x = layer(x)
        return x
