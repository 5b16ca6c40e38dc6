"""Convolutional encoder for 2-D observation groups (``rsl_rl/modules/cnn.py``); PyTorch path only."""

from __future__ import annotations

import math

import torch
from torch import nn

from ..utils.utils import get_param, resolve_nn_activation

_PADDING_MODES = ("zeros", "reflect", "replicate", "circular")


def _same_padding(hw: tuple[int, int], k: int, s: int, d: int) -> tuple[int, int]:
    def one(x: int) -> int:
        return math.ceil((s * math.floor(x / s) - x - s + d * (k - 1) + 1) / 2)

    return one(hw[0]), one(hw[1])


def _out_hw(hw: tuple[int, int], k: int, s: int, d: int, p: tuple[int, int], pooled: bool = False) -> tuple[int, int]:
    h = math.floor((hw[0] + 2 * p[0] - d * (k - 1) - 1) / s + 1)
    w = math.floor((hw[1] + 2 * p[1] - d * (k - 1) - 1) / s + 1)
    if pooled:
        h, w = math.ceil(h / 2), math.ceil(w / 2)
    return h, w


class CNN(nn.Sequential):
    """Conv2d stack with optional batch/layer norm, max pooling, global pooling and flattening."""

    def __init__(
        self,
        input_dim: tuple[int, int],
        input_channels: int,
        output_channels: tuple[int, ...] | list[int],
        kernel_size: int | tuple[int, ...] | list[int],
        stride: int | tuple[int, ...] | list[int] = 1,
        dilation: int | tuple[int, ...] | list[int] = 1,
        padding: str = "none",
        norm: str | tuple[str] | list[str] = "none",
        activation: str = "elu",
        max_pool: bool | tuple[bool] | list[bool] = False,
        global_pool: str = "none",
        flatten: bool = True,
    ) -> None:
        super().__init__()
        act = resolve_nn_activation(activation)
        layers: list[nn.Module] = []
        channels = input_channels
        hw = tuple(input_dim)
        for i, out_c in enumerate(output_channels):
            k, s, d = get_param(kernel_size, i), get_param(stride, i), get_param(dilation, i)
            p = _same_padding(hw, k, s, d) if padding in _PADDING_MODES else (0, 0)
            layers.append(nn.Conv2d(channels, out_c, kernel_size=k, stride=s, padding=p, dilation=d,
                                    padding_mode=padding if padding in _PADDING_MODES else "zeros"))
            n = get_param(norm, i)
            if n == "batch":
                layers.append(nn.BatchNorm2d(out_c))
            elif n == "layer":
                oh, ow = _out_hw(hw, k, s, d, p)
                layers.append(nn.LayerNorm([out_c, oh, ow]))
            elif n != "none":
                raise ValueError(f"Unsupported normalization type: {n}. Supported types are 'none', 'batch', and 'layer'.")
            layers.append(act)
            pooled = bool(get_param(max_pool, i))
            if pooled:
                layers.append(nn.MaxPool2d(kernel_size=3, stride=2, padding=1))
            channels = out_c
            hw = _out_hw(hw, k, s, d, p, pooled)
        if global_pool == "max":
            layers.append(nn.AdaptiveMaxPool2d((1, 1)))
            hw = (1, 1)
        elif global_pool == "avg":
            layers.append(nn.AdaptiveAvgPool2d((1, 1)))
            hw = (1, 1)
        elif global_pool != "none":
            raise ValueError(
                f"Unsupported global pooling type: {global_pool}. Supported types are 'none', 'max', and 'avg'."
            )
        if flatten:
            layers.append(nn.Flatten(start_dim=1))
        self._output_channels = None if flatten else channels
        self._output_dim = channels * hw[0] * hw[1] if flatten else hw
        for i, layer in enumerate(layers):
            self.add_module(str(i), layer)

    @property
    def output_channels(self) -> int | None:
        return self._output_channels

    @property
    def output_dim(self) -> tuple[int, int] | int:
        return self._output_dim

    def init_weights(self) -> None:
        for m in self:
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight)
                nn.init.zeros_(m.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self:
            x = layer(x)
        return x
