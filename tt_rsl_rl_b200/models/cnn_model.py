"""CNN actor/critic model (``rsl_rl/models/cnn_model.py``): CNN encoders for 2-D groups plus normalised 1-D groups
feeding an MLP. PyTorch path only (not part of the GPU benchmark configurations)."""

from __future__ import annotations

import copy
from typing import Any

import torch
import torch.nn as nn

from ..modules import CNN, HiddenState
from .mlp_model import MLPModel, _deterministic_head


class CNNModel(MLPModel):
    def __init__(
        self,
        obs,
        obs_groups: dict[str, list[str]],
        obs_set: str,
        output_dim: int,
        hidden_dims: tuple[int, ...] | list[int] = (256, 256, 256),
        activation: str = "elu",
        obs_normalization: bool = False,
        distribution_cfg: dict | None = None,
        cnn_cfg: dict[str, dict] | dict[str, Any] | None = None,
        cnns: nn.ModuleDict | dict[str, nn.Module] | None = None,
    ) -> None:
        self._get_obs_dim(obs, obs_groups, obs_set)
        if cnns is not None:
            if set(cnns.keys()) != set(self.obs_groups_2d):
                raise ValueError("The 2D observations must be identical for all models sharing CNN encoders.")
            print("Sharing CNN encoders between models, the CNN configurations of the receiving model are ignored.")
        else:
            if cnn_cfg is None:
                raise ValueError("CNN configurations must be provided if CNNs are not shared.")
            if not all(isinstance(v, dict) for v in cnn_cfg.values()):
                cnn_cfg = {g: cnn_cfg for g in self.obs_groups_2d}
            if len(cnn_cfg) != len(self.obs_groups_2d):
                raise ValueError("The number of CNN configurations must match the number of 2D observation groups.")
            cnns = {
                g: CNN(input_dim=self.obs_dims_2d[i], input_channels=self.obs_channels_2d[i], **cnn_cfg[g])
                for i, g in enumerate(self.obs_groups_2d)
            }
        self.cnn_latent_dim = 0
        for cnn in cnns.values():
            if cnn.output_channels is not None:
                raise ValueError("The output of the CNN must be flattened before passing it to the MLP.")
            self.cnn_latent_dim += int(cnn.output_dim)
        super().__init__(obs, obs_groups, obs_set, output_dim, hidden_dims, activation, obs_normalization,
                         distribution_cfg)
        self.cnns = cnns if isinstance(cnns, nn.ModuleDict) else nn.ModuleDict(cnns)

    def get_latent(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None) -> torch.Tensor:
        latent_cnn = torch.cat([self.cnns[g](obs[g]) for g in self.obs_groups_2d], dim=-1)
        if not self.obs_groups:
            return latent_cnn
        return torch.cat([super().get_latent(obs), latent_cnn], dim=-1)

    def as_jit(self) -> nn.Module:
        return _TorchCNNModel(self)

    def as_onnx(self) -> nn.Module:
        return _OnnxCNNModel(self)

    def _get_obs_dim(self, obs, obs_groups: dict[str, list[str]], obs_set: str) -> tuple[list[str], int]:
        groups_1d, dims_2d, channels_2d, groups_2d = [], [], [], []
        dim_1d = 0
        for g in obs_groups[obs_set]:
            shape = obs[g].shape
            if len(shape) == 4:
                groups_2d.append(g)
                dims_2d.append(tuple(shape[2:4]))
                channels_2d.append(shape[1])
            elif len(shape) == 2:
                groups_1d.append(g)
                dim_1d += shape[-1]
            else:
                raise ValueError(f"Invalid observation shape for {g}: {shape}")
        if not groups_2d:
            raise ValueError("No 2D observations are provided. If this is intentional, use the MLP model instead.")
        self.obs_dims_2d = dims_2d
        self.obs_channels_2d = channels_2d
        self.obs_groups_2d = groups_2d
        return groups_1d, dim_1d

    def _get_latent_dim(self) -> int:
        return self.obs_dim + self.cnn_latent_dim


class _TorchCNNModel(nn.Module):
    def __init__(self, model: CNNModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.cnns = nn.ModuleList([copy.deepcopy(model.cnns[g]) for g in model.obs_groups_2d])
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)

    def forward(self, obs_1d: torch.Tensor, obs_2d: list[torch.Tensor]) -> torch.Tensor:
        parts = [self.obs_normalizer(obs_1d)]
        for i, cnn in enumerate(self.cnns):
            parts.append(cnn(obs_2d[i]))
        return self.deterministic_output(self.mlp(torch.cat(parts, dim=-1)))

    @torch.jit.export
    def reset(self) -> None:
        pass


class _OnnxCNNModel(nn.Module):
    def __init__(self, model: CNNModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.cnns = nn.ModuleList([copy.deepcopy(model.cnns[g]) for g in model.obs_groups_2d])
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)
        self.obs_groups_2d = model.obs_groups_2d
        self.obs_dims_2d = model.obs_dims_2d
        self.obs_channels_2d = model.obs_channels_2d
        self.obs_dim_1d = model.obs_dim

    def forward(self, obs_1d: torch.Tensor, *obs_2d: torch.Tensor) -> torch.Tensor:
        parts = [self.obs_normalizer(obs_1d)]
        for i, cnn in enumerate(self.cnns):
            parts.append(cnn(obs_2d[i]))
        return self.deterministic_output(self.mlp(torch.cat(parts, dim=-1)))

    def get_dummy_inputs(self) -> tuple[torch.Tensor, ...]:
        dummies = [torch.zeros(1, self.obs_dim_1d)]
        for (h, w), c in zip(self.obs_dims_2d, self.obs_channels_2d):
            dummies.append(torch.zeros(1, c, h, w))
        return tuple(dummies)

    @property
    def input_names(self) -> list[str]:
        return ["obs", *self.obs_groups_2d]

    @property
    def output_names(self) -> list[str]:
        return ["actions"]
