"""Feed-forward actor / critic model.

Public interface of rsl_rl's ``MLPModel`` (``rsl_rl/models/mlp_model.py``): the constructor arguments, the module
tree ``obs_normalizer`` / ``distribution`` / ``mlp`` (so state dicts and checkpoints are interchangeable), the
recurrent no-op interface and the distribution accessors that the algorithms call.

Design of this package:

* :class:`ObservationLayout` resolves an observation set once into its flat groups (``[B, D]``, concatenated and
  optionally normalised) and its image groups (``[B, C, H, W]``, for encoder models); the model families differ only
  in which layouts they accept and in the encoder that turns observations into the MLP's input (the *latent*).
* Construction happens in a fixed order that the subclasses hook into: encoders that draw their initial weights
  before the MLP (CNN encoders), normaliser, distribution, MLP, then encoders registered after it (the recurrent
  layer). The order decides both the random draws of the initial weights and the order of ``parameters()``, which
  indexes the optimizer state in a checkpoint; it is rsl_rl's, so seeded models and optimizer states agree with it.
* Export: one TorchScript module and one ONNX module for every feed-forward model (with or without image encoders).

On CUDA the fused engines run the MLP through sm_100a kernels on these same parameters; ``forward`` here is the
PyTorch definition, used on the CPU, for export and for evaluation.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn as nn

from ..modules import MLP, EmpiricalNormalization, HiddenState
from ..modules.distribution import Distribution
from ..utils.utils import resolve_class, unpad_trajectories


@dataclass
class ObservationLayout:
    """Groups of one observation set: flat ``[B, D]`` groups and image ``[B, C, H, W]`` groups, in config order."""

    flat: list[str] = field(default_factory=list)
    flat_dim: int = 0
    images: list[str] = field(default_factory=list)
    image_hw: list[tuple[int, int]] = field(default_factory=list)
    image_channels: list[int] = field(default_factory=list)

    @classmethod
    def of(cls, obs, groups: list[str], images: bool) -> "ObservationLayout":
        out = cls()
        for g in groups:
            shape = obs[g].shape
            if len(shape) == 2:
                out.flat.append(g)
                out.flat_dim += shape[-1]
            elif images and len(shape) == 4:
                out.images.append(g)
                out.image_hw.append(tuple(shape[2:4]))
                out.image_channels.append(shape[1])
            elif images:
                raise ValueError(f"observation group '{g}' has shape {tuple(shape)}: expected [B, D] or [B, C, H, W]")
            else:
                raise ValueError(f"observation group '{g}' has shape {tuple(shape)}: this model reads [B, D] groups "
                                 "only (use CNNModel for images)")
        return out


class MLPModel(nn.Module):
    """Observation groups -> concatenation -> optional empirical normalisation -> MLP -> optional distribution."""

    is_recurrent: bool = False
    _reads_images: bool = False

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
        **encoder_cfg,
    ) -> None:
        super().__init__()
        layout = ObservationLayout.of(obs, obs_groups[obs_set], images=self._reads_images)
        self.obs_groups, self.obs_dim = layout.flat, layout.flat_dim
        early = self._encoders_before_head(layout, **encoder_cfg)
        self.obs_normalization = obs_normalization
        self.obs_normalizer = EmpiricalNormalization(self.obs_dim) if obs_normalization else nn.Identity()
        self.distribution: Distribution | None = None
        if distribution_cfg is not None:
            dist_cls, dist_kwargs = resolve_class(distribution_cfg)
            self.distribution = dist_cls(output_dim, **dist_kwargs)
        self.output_dim = output_dim
        self.hidden_dims = list(hidden_dims)
        self.activation = activation
        head_out = output_dim if self.distribution is None else self.distribution.input_dim
        self.mlp = MLP(self._get_latent_dim(), head_out, hidden_dims, activation)
        if self.distribution is not None:
            self.distribution.init_mlp_weights(self.mlp)
        self._encoders_after_head(layout, early, **encoder_cfg)

    # ---- construction hooks of the model families ----------------------------------------------------------------------
    def _encoders_before_head(self, layout: ObservationLayout, **cfg):
        """Build encoders whose initial weights are drawn before the MLP's; returns what the later hook registers."""
        if cfg:
            raise TypeError(f"unexpected arguments for {type(self).__name__}: {sorted(cfg)}")
        return None

    def _encoders_after_head(self, layout: ObservationLayout, early, **cfg) -> None:
        """Register encoders as submodules after the MLP (their parameters come after the MLP's)."""

    def _get_latent_dim(self) -> int:
        return self.obs_dim

    # ---- forward ----------------------------------------------------------------------------------------------------
    def forward(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None,
                stochastic_output: bool = False) -> torch.Tensor:
        """MLP output, or with a distribution its deterministic output (default) or a sample of it."""
        if masks is not None and not self.is_recurrent:  # padded trajectory batches of a recurrent algorithm
            obs = unpad_trajectories(obs, masks)
        out = self.mlp(self.get_latent(obs, masks, hidden_state))
        dist = self.distribution
        if dist is None:
            return out
        if not stochastic_output:
            return dist.deterministic_output(out)
        dist.update(out)
        return dist.sample()

    def concat_obs(self, obs) -> torch.Tensor:
        """The flat observation groups of this model side by side."""
        return torch.cat([obs[g] for g in self.obs_groups], dim=-1)

    def get_latent(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None) -> torch.Tensor:
        return self.obs_normalizer(self.concat_obs(obs))

    # ---- recurrent interface (nothing to do without a recurrent layer) --------------------------------------------
    def reset(self, dones: torch.Tensor | None = None, hidden_state: HiddenState = None) -> None:
        return None

    def get_hidden_state(self) -> HiddenState:
        return None

    def detach_hidden_state(self, dones: torch.Tensor | None = None) -> None:
        return None

    # ---- distribution accessors -------------------------------------------------------------------------------------
    output_mean = property(lambda self: self.distribution.mean, doc="Mean of the current output distribution.")
    output_std = property(lambda self: self.distribution.std, doc="Std of the current output distribution.")
    output_entropy = property(lambda self: self.distribution.entropy, doc="Entropy of the current distribution.")
    output_distribution_params = property(lambda self: self.distribution.params,
                                          doc="Parameters of the current output distribution.")

    def get_output_log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        return self.distribution.log_prob(outputs)

    def get_kl_divergence(self, old_params: tuple[torch.Tensor, ...],
                          new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        return self.distribution.kl_divergence(old_params, new_params)

    # ---- normalisation ----------------------------------------------------------------------------------------------
    def update_normalization(self, obs) -> None:
        """Fold a batch of observations into the running statistics of the normaliser."""
        if self.obs_normalization and self.obs_groups:
            self.obs_normalizer.update(self.concat_obs(obs))

    # ---- export -----------------------------------------------------------------------------------------------------
    def _export_parts(self) -> tuple[nn.Module, nn.ModuleList, nn.Module, nn.Module]:
        """Copies of (normaliser, image encoders, MLP, deterministic output head) for an exported module."""
        head = nn.Identity() if self.distribution is None else self.distribution.as_deterministic_output_module()
        return copy.deepcopy(self.obs_normalizer), nn.ModuleList(), copy.deepcopy(self.mlp), head

    def as_jit(self) -> nn.Module:
        return ScriptedFeedForward(self)

    def as_onnx(self) -> nn.Module:
        return OnnxFeedForward(self)


class ScriptedFeedForward(nn.Module):
    """TorchScript policy of a feed-forward model: ``forward(obs, images=None)`` with the flat observations already
    concatenated, and for encoder models the image groups as a list in configuration order."""

    def __init__(self, model: MLPModel) -> None:
        super().__init__()
        self.obs_normalizer, self.encoders, self.mlp, self.deterministic_output = model._export_parts()

    def forward(self, x: torch.Tensor, images: Optional[List[torch.Tensor]] = None) -> torch.Tensor:
        parts = [self.obs_normalizer(x)]
        if images is not None:
            for i, enc in enumerate(self.encoders):
                parts.append(enc(images[i]))
        latent = parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)
        return self.deterministic_output(self.mlp(latent))

    @torch.jit.export
    def reset(self) -> None:
        pass


class OnnxFeedForward(nn.Module):
    """ONNX policy of a feed-forward model: inputs ``obs`` and one input per image group."""

    is_recurrent: bool = False

    def __init__(self, model: MLPModel) -> None:
        super().__init__()
        self.obs_normalizer, self.encoders, self.mlp, self.deterministic_output = model._export_parts()
        self.input_size = model.obs_dim
        self.image_groups = list(getattr(model, "obs_groups_2d", []))
        self.image_shapes = [(c, *hw) for c, hw in zip(getattr(model, "obs_channels_2d", []),
                                                        getattr(model, "obs_dims_2d", []))]

    def forward(self, x: torch.Tensor, *images: torch.Tensor) -> torch.Tensor:
        parts = [self.obs_normalizer(x)] + [enc(img) for enc, img in zip(self.encoders, images)]
        latent = parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)
        return self.deterministic_output(self.mlp(latent))

    def get_dummy_inputs(self) -> tuple[torch.Tensor, ...]:
        return (torch.zeros(1, self.input_size), *[torch.zeros(1, *s) for s in self.image_shapes])

    @property
    def input_names(self) -> list[str]:
        return ["obs", *self.image_groups]

    @property
    def output_names(self) -> list[str]:
        return ["actions"]
