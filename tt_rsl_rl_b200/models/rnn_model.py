"""Recurrent actor / critic model: normaliser -> GRU or LSTM -> MLP head.

Public interface of rsl_rl's ``RNNModel`` (``rsl_rl/models/rnn_model.py``): constructor arguments, the module tree
(``rnn.rnn.weight_ih_l0`` ... after the MLP, so checkpoints and optimizer states line up), the hidden-state
interface, and TorchScript / ONNX exports that carry the hidden state.

Here the recurrent layer is the encoder of :class:`MLPModel`'s construction scheme, registered after the MLP; the
latent is the recurrent output of the normalised observations. On CUDA the recurrent PPO engine runs the cell
(rollout) and the full-sequence forward / BPTT through sm_100a kernels with these same parameters.
"""

from __future__ import annotations

import copy

import torch
import torch.nn as nn

from ..modules import RNN, HiddenState
from .mlp_model import MLPModel, ObservationLayout


class RNNModel(MLPModel):
    is_recurrent: bool = True

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
        rnn_type: str = "lstm",
        rnn_hidden_dim: int = 256,
        rnn_num_layers: int = 1,
    ) -> None:
        self.latent_dim = rnn_hidden_dim  # the MLP reads the recurrent output
        super().__init__(obs, obs_groups, obs_set, output_dim, hidden_dims, activation, obs_normalization,
                         distribution_cfg, rnn_type=rnn_type, rnn_hidden_dim=rnn_hidden_dim,
                         rnn_num_layers=rnn_num_layers)

    def _encoders_before_head(self, layout: ObservationLayout, **cfg):
        return None

    def _encoders_after_head(self, layout: ObservationLayout, early, rnn_type: str, rnn_hidden_dim: int,
                             rnn_num_layers: int) -> None:
        self.rnn_type = rnn_type.lower()
        self.rnn = RNN(self.obs_dim, rnn_hidden_dim, rnn_num_layers, rnn_type)

    def _get_latent_dim(self) -> int:
        return self.latent_dim

    def get_latent(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None) -> torch.Tensor:
        """Recurrent output of the normalised observations: one step in rollout mode (``masks`` None, internal
        state), or whole padded trajectories from ``hidden_state`` in batch mode."""
        return self.rnn(super().get_latent(obs), masks, hidden_state).squeeze(0)

    # ---- hidden state -------------------------------------------------------------------------------------------------
    def reset(self, dones: torch.Tensor | None = None, hidden_state: HiddenState = None) -> None:
        self.rnn.reset(dones, hidden_state)

    def get_hidden_state(self) -> HiddenState:
        return self.rnn.hidden_state

    def detach_hidden_state(self, dones: torch.Tensor | None = None) -> None:
        self.rnn.detach_hidden_state(dones)

    # ---- export -------------------------------------------------------------------------------------------------------
    def _recurrent_copy(self) -> nn.Module:
        cell = self.rnn.rnn
        if not isinstance(cell, (nn.GRU, nn.LSTM)):
            raise NotImplementedError(f"no export for recurrent layer {type(cell).__name__}")
        return copy.deepcopy(cell)

    def as_jit(self) -> nn.Module:
        return ScriptedLSTM(self) if isinstance(self.rnn.rnn, nn.LSTM) else ScriptedGRU(self)

    def as_onnx(self) -> nn.Module:
        return OnnxRecurrent(self)


class _ScriptedRecurrentBase(nn.Module):
    """Parts shared by the stateful TorchScript policies: one observation row per call, state kept in buffers."""

    def __init__(self, model: RNNModel) -> None:
        super().__init__()
        self.obs_normalizer, _, self.mlp, self.deterministic_output = model._export_parts()
        self.rnn = model._recurrent_copy()
        self.register_buffer("hidden_state", torch.zeros(self.rnn.num_layers, 1, self.rnn.hidden_size))

    def _head(self, y: torch.Tensor) -> torch.Tensor:
        return self.deterministic_output(self.mlp(y.squeeze(0)))


class ScriptedGRU(_ScriptedRecurrentBase):
    def __init__(self, model: RNNModel) -> None:
        super().__init__(model)
        self.rnn.cpu()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y, h = self.rnn(self.obs_normalizer(x).unsqueeze(0), self.hidden_state)
        self.hidden_state[:] = h
        return self._head(y)

    @torch.jit.export
    def reset(self) -> None:
        self.hidden_state[:] = 0.0


class ScriptedLSTM(_ScriptedRecurrentBase):
    def __init__(self, model: RNNModel) -> None:
        super().__init__(model)
        self.register_buffer("cell_state", torch.zeros(self.rnn.num_layers, 1, self.rnn.hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y, (h, c) = self.rnn(self.obs_normalizer(x).unsqueeze(0), (self.hidden_state, self.cell_state))
        self.hidden_state[:] = h
        self.cell_state[:] = c
        return self._head(y)

    @torch.jit.export
    def reset(self) -> None:
        self.hidden_state[:] = 0.0
        self.cell_state[:] = 0.0


class OnnxRecurrent(nn.Module):
    """ONNX policy with explicit state: ``(obs, h_in[, c_in]) -> (actions, h_out[, c_out])``."""

    is_recurrent: bool = True

    def __init__(self, model: RNNModel) -> None:
        super().__init__()
        self.obs_normalizer, _, self.mlp, self.deterministic_output = model._export_parts()
        self.rnn = model._recurrent_copy()
        self.rnn_type = "lstm" if isinstance(self.rnn, nn.LSTM) else "gru"
        self.input_size = model.obs_dim
        self.hidden_size = self.rnn.hidden_size
        self.num_layers = self.rnn.num_layers

    def forward(self, obs: torch.Tensor, h_in: torch.Tensor, c_in: torch.Tensor | None = None):
        x = self.obs_normalizer(obs).unsqueeze(0)
        if self.rnn_type == "lstm":
            y, (h, c) = self.rnn(x, (h_in, c_in))
        else:
            (y, h), c = self.rnn(x, h_in), None
        return self.deterministic_output(self.mlp(y.squeeze(0))), h, c

    def _state(self) -> torch.Tensor:
        return torch.zeros(self.num_layers, 1, self.hidden_size)

    def get_dummy_inputs(self) -> tuple[torch.Tensor, ...]:
        inputs = (torch.zeros(1, self.input_size), self._state())
        return inputs + (self._state(),) if self.rnn_type == "lstm" else inputs

    @property
    def input_names(self) -> list[str]:
        return ["obs", "h_in", "c_in"] if self.rnn_type == "lstm" else ["obs", "h_in"]

    @property
    def output_names(self) -> list[str]:
        return ["actions", "h_out", "c_out"] if self.rnn_type == "lstm" else ["actions", "h_out"]
