"""MLP actor/critic model (``rsl_rl/models/mlp_model.py``): observation groups -> concat -> optional empirical
normalisation -> MLP -> optional output distribution.

The module tree (``obs_normalizer``, ``mlp``, ``distribution``) and parameter names match rsl_rl, so state dicts are
interchangeable. On CUDA the PPO engine (``tt_rsl_rl_b200.engine``) runs this model through fused sm_100a kernels using
the same parameters; the ``forward`` here is the PyTorch definition used on CPU, for export and for evaluation.
"""

from __future__ import annotations

import copy

import torch
import torch.nn as nn

from ..modules import MLP, EmpiricalNormalization, HiddenState
from ..modules.distribution import Distribution
from ..utils.utils import resolve_class, unpad_trajectories


class MLPModel(nn.Module):
    is_recurrent: bool = False

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
    ) -> None:
        super().__init__()
        self.obs_groups, self.obs_dim = self._get_obs_dim(obs, obs_groups, obs_set)
        self.obs_normalization = obs_normalization
        self.obs_normalizer = EmpiricalNormalization(self.obs_dim) if obs_normalization else nn.Identity()
        self.output_dim = output_dim
        self.hidden_dims = list(hidden_dims)
        self.activation = activation
        if distribution_cfg is not None:
            dist_class, dist_kwargs = resolve_class(distribution_cfg)
            self.distribution: Distribution | None = dist_class(output_dim, **dist_kwargs)
            head_dim = self.distribution.input_dim
        else:
            self.distribution = None
            head_dim = output_dim
        self.mlp = MLP(self._get_latent_dim(), head_dim, hidden_dims, activation)
        if self.distribution is not None:
            self.distribution.init_mlp_weights(self.mlp)

    # ---- forward ----------------------------------------------------------------------------------------------------
    def forward(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None,
                stochastic_output: bool = False) -> torch.Tensor:
        if masks is not None and not self.is_recurrent:
            obs = unpad_trajectories(obs, masks)
        out = self.mlp(self.get_latent(obs, masks, hidden_state))
        if self.distribution is None:
            return out
        if stochastic_output:
            self.distribution.update(out)
            return self.distribution.sample()
        return self.distribution.deterministic_output(out)

    def get_latent(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None) -> torch.Tensor:
        return self.obs_normalizer(self.concat_obs(obs))

    def concat_obs(self, obs) -> torch.Tensor:
        """Concatenation of this model's observation groups along the last dimension."""
        return torch.cat([obs[g] for g in self.obs_groups], dim=-1)

    # ---- recurrent interface (no-ops for MLPs) ------------------------------------------------------------------------
    def reset(self, dones: torch.Tensor | None = None, hidden_state: HiddenState = None) -> None:
        pass

    def get_hidden_state(self) -> HiddenState:
        return None

    def detach_hidden_state(self, dones: torch.Tensor | None = None) -> None:
        pass

    # ---- distribution accessors -------------------------------------------------------------------------------------
    @property
    def output_mean(self) -> torch.Tensor:
        return self.distribution.mean

    @property
    def output_std(self) -> torch.Tensor:
        return self.distribution.std

    @property
    def output_entropy(self) -> torch.Tensor:
        return self.distribution.entropy

    @property
    def output_distribution_params(self) -> tuple[torch.Tensor, ...]:
        return self.distribution.params

    def get_output_log_prob(self, outputs: torch.Tensor) -> torch.Tensor:
        return self.distribution.log_prob(outputs)

    def get_kl_divergence(self, old_params: tuple[torch.Tensor, ...],
                          new_params: tuple[torch.Tensor, ...]) -> torch.Tensor:
        return self.distribution.kl_divergence(old_params, new_params)

    # ---- export -----------------------------------------------------------------------------------------------------
    def as_jit(self) -> nn.Module:
        return _TorchMLPModel(self)

    def as_onnx(self) -> nn.Module:
        return _OnnxMLPModel(self)

    # ---- normalisation ----------------------------------------------------------------------------------------------
    def update_normalization(self, obs) -> None:
        if self.obs_normalization and self.obs_groups:
            self.obs_normalizer.update(self.concat_obs(obs))

    # ---- helpers ----------------------------------------------------------------------------------------------------
    def _get_obs_dim(self, obs, obs_groups: dict[str, list[str]], obs_set: str) -> tuple[list[str], int]:
        groups = obs_groups[obs_set]
        dim = 0
        for g in groups:
            if len(obs[g].shape) != 2:
                raise ValueError(f"The MLP model only supports 1D observations, got shape {obs[g].shape} for '{g}'.")
            dim += obs[g].shape[-1]
        return groups, dim

    def _get_latent_dim(self) -> int:
        return self.obs_dim


def _deterministic_head(model: MLPModel) -> nn.Module:
    if model.distribution is not None:
        return model.distribution.as_deterministic_output_module()
    return nn.Identity()


class _TorchMLPModel(nn.Module):
    """TorchScript export: normalised observations -> MLP -> deterministic output."""

    def __init__(self, model: MLPModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.deterministic_output(self.mlp(self.obs_normalizer(x)))

    @torch.jit.export
    def reset(self) -> None:
        pass


class _OnnxMLPModel(nn.Module):
    """ONNX export wrapper with named inputs/outputs and dummy inputs."""

    is_recurrent: bool = False

    def __init__(self, model: MLPModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)
        self.input_size = model.obs_dim

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.deterministic_output(self.mlp(self.obs_normalizer(x)))

    def get_dummy_inputs(self) -> tuple[torch.Tensor]:
        return (torch.zeros(1, self.input_size),)

    @property
    def input_names(self) -> list[str]:
        return ["obs"]

    @property
    def output_names(self) -> list[str]:
        return ["actions"]
