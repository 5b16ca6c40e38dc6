"""Actor / critic model with convolutional encoders for image observations.

Public interface of rsl_rl's ``CNNModel`` (``rsl_rl/models/cnn_model.py``): image groups ``[B, C, H, W]`` each go
through a CNN encoder (configured per group, one configuration for all, or modules shared with another model), flat
groups are concatenated and optionally normalised, and the MLP reads ``[flat latent, encoder outputs]``.

Here the encoders are built by the first hook of :class:`MLPModel`'s construction scheme (their initial weights are
drawn before the MLP's) and registered by the second one (their parameters follow the MLP's). PyTorch path only.
"""

from __future__ import annotations

from typing import Any

import copy

import torch
import torch.nn as nn

from ..modules import CNN, HiddenState
from .mlp_model import MLPModel, ObservationLayout


class CNNModel(MLPModel):
    _reads_images: bool = True

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
        super().__init__(obs, obs_groups, obs_set, output_dim, hidden_dims, activation, obs_normalization,
                         distribution_cfg, cnn_cfg=cnn_cfg, cnns=cnns)

    def _encoders_before_head(self, layout: ObservationLayout, cnn_cfg=None, cnns=None):
        if not layout.images:
            raise ValueError("CNNModel needs at least one image observation group [B, C, H, W]; use MLPModel "
                             "for flat observations only")
        self.obs_groups_2d = layout.images
        self.obs_dims_2d = layout.image_hw
        self.obs_channels_2d = layout.image_channels
        if cnns is not None:  # encoders shared with another model (e.g. actor and critic)
            if set(cnns.keys()) != set(layout.images):
                raise ValueError("models sharing CNN encoders must read the same image groups")
            print("Sharing CNN encoders between models, the CNN configurations of the receiving model are ignored.")
            encoders = dict(cnns)
        else:
            encoders = {g: CNN(input_dim=hw, input_channels=c, **cfg)
                        for g, hw, c, cfg in zip(layout.images, layout.image_hw, layout.image_channels,
                                                 self._per_group_cfg(layout, cnn_cfg))}
        widths = []
        for enc in encoders.values():
            if enc.output_channels is not None:
                raise ValueError("a CNN encoder must end flattened (no output channels) to feed the MLP")
            widths.append(int(enc.output_dim))
        self.cnn_latent_dim = sum(widths)
        return cnns if isinstance(cnns, nn.ModuleDict) else encoders

    @staticmethod
    def _per_group_cfg(layout: ObservationLayout, cnn_cfg) -> list[dict]:
        """One configuration per image group: a dict of per-group dicts, or one configuration for all groups."""
        if cnn_cfg is None:
            raise ValueError("cnn_cfg is required unless CNN encoders are shared (cnns=...)")
        if not all(isinstance(v, dict) for v in cnn_cfg.values()):
            return [cnn_cfg] * len(layout.images)
        if len(cnn_cfg) != len(layout.images):
            raise ValueError(f"cnn_cfg has {len(cnn_cfg)} entries for {len(layout.images)} image groups")
        return [cnn_cfg[g] for g in layout.images]

    def _encoders_after_head(self, layout: ObservationLayout, early, cnn_cfg=None, cnns=None) -> None:
        self.cnns = early if isinstance(early, nn.ModuleDict) else nn.ModuleDict(early)

    def _get_latent_dim(self) -> int:
        return self.obs_dim + self.cnn_latent_dim

    def get_latent(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None) -> torch.Tensor:
        encoded = torch.cat([self.cnns[g](obs[g]) for g in self.obs_groups_2d], dim=-1)
        if not self.obs_groups:
            return encoded
        return torch.cat([super().get_latent(obs), encoded], dim=-1)

    def _export_parts(self):
        norm, _, mlp, head = super()._export_parts()
        return norm, nn.ModuleList([copy.deepcopy(self.cnns[g]) for g in self.obs_groups_2d]), mlp, head
