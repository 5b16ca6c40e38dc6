"""Recurrent actor/critic model (``rsl_rl/models/rnn_model.py``): normaliser -> GRU/LSTM -> MLP head.

On CUDA the recurrent PPO path runs the cell (rollout) and the full-sequence forward/BPTT through the framework's
sm_100a kernels with these same parameters (``rnn.rnn.weight_ih_l0`` ...).
"""

from __future__ import annotations

import copy

import torch
import torch.nn as nn

from ..modules import RNN, HiddenState
from .mlp_model import MLPModel, _deterministic_head


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
        self.latent_dim = rnn_hidden_dim
        super().__init__(obs, obs_groups, obs_set, output_dim, hidden_dims, activation, obs_normalization,
                         distribution_cfg)
        self.rnn_type = rnn_type.lower()
        self.rnn = RNN(self.obs_dim, rnn_hidden_dim, rnn_num_layers, rnn_type)

    def get_latent(self, obs, masks: torch.Tensor | None = None, hidden_state: HiddenState = None) -> torch.Tensor:
        x = super().get_latent(obs)
        return self.rnn(x, masks, hidden_state).squeeze(0)

    def reset(self, dones: torch.Tensor | None = None, hidden_state: HiddenState = None) -> None:
        self.rnn.reset(dones, hidden_state)

    def get_hidden_state(self) -> HiddenState:
        return self.rnn.hidden_state

    def detach_hidden_state(self, dones: torch.Tensor | None = None) -> None:
        self.rnn.detach_hidden_state(dones)

    def as_jit(self) -> nn.Module:
        if isinstance(self.rnn.rnn, nn.LSTM):
            return _TorchLSTMModel(self)
        if isinstance(self.rnn.rnn, nn.GRU):
            return _TorchGRUModel(self)
        raise NotImplementedError(f"Unsupported RNN type: {type(self.rnn.rnn)}")

    def as_onnx(self) -> nn.Module:
        return _OnnxRNNModel(self)

    def _get_latent_dim(self) -> int:
        return self.latent_dim


class _TorchGRUModel(nn.Module):
    def __init__(self, model: RNNModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.rnn = copy.deepcopy(model.rnn.rnn)
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)
        self.rnn.cpu()
        self.register_buffer("hidden_state", torch.zeros(self.rnn.num_layers, 1, self.rnn.hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.obs_normalizer(x)
        y, h = self.rnn(x.unsqueeze(0), self.hidden_state)
        self.hidden_state[:] = h
        return self.deterministic_output(self.mlp(y.squeeze(0)))

    @torch.jit.export
    def reset(self) -> None:
        self.hidden_state[:] = 0.0


class _TorchLSTMModel(nn.Module):
    def __init__(self, model: RNNModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.rnn = copy.deepcopy(model.rnn.rnn)
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)
        self.register_buffer("hidden_state", torch.zeros(self.rnn.num_layers, 1, self.rnn.hidden_size))
        self.register_buffer("cell_state", torch.zeros(self.rnn.num_layers, 1, self.rnn.hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.obs_normalizer(x)
        y, (h, c) = self.rnn(x.unsqueeze(0), (self.hidden_state, self.cell_state))
        self.hidden_state[:] = h
        self.cell_state[:] = c
        return self.deterministic_output(self.mlp(y.squeeze(0)))

    @torch.jit.export
    def reset(self) -> None:
        self.hidden_state[:] = 0.0
        self.cell_state[:] = 0.0


class _OnnxRNNModel(nn.Module):
    is_recurrent: bool = True

    def __init__(self, model: RNNModel) -> None:
        super().__init__()
        self.obs_normalizer = copy.deepcopy(model.obs_normalizer)
        self.rnn = copy.deepcopy(model.rnn.rnn)
        self.mlp = copy.deepcopy(model.mlp)
        self.deterministic_output = _deterministic_head(model)
        if isinstance(self.rnn, nn.LSTM):
            self.rnn_type = "lstm"
        elif isinstance(self.rnn, nn.GRU):
            self.rnn_type = "gru"
        else:
            raise NotImplementedError(f"Unsupported RNN type: {type(self.rnn)}")
        self.input_size = model.obs_dim
        self.hidden_size = self.rnn.hidden_size
        self.num_layers = self.rnn.num_layers

    def forward(self, obs: torch.Tensor, h_in: torch.Tensor, c_in: torch.Tensor | None = None):
        x = self.obs_normalizer(obs)
        if self.rnn_type == "lstm":
            y, (h, c) = self.rnn(x.unsqueeze(0), (h_in, c_in))
            return self.deterministic_output(self.mlp(y.squeeze(0))), h, c
        y, h = self.rnn(x.unsqueeze(0), h_in)
        return self.deterministic_output(self.mlp(y.squeeze(0))), h, None

    def get_dummy_inputs(self) -> tuple[torch.Tensor, ...]:
        obs = torch.zeros(1, self.input_size)
        h = torch.zeros(self.num_layers, 1, self.hidden_size)
        if self.rnn_type == "lstm":
            return (obs, h, torch.zeros(self.num_layers, 1, self.hidden_size))
        return (obs, h)

    @property
    def input_names(self) -> list[str]:
        return ["obs", "h_in", "c_in"] if self.rnn_type == "lstm" else ["obs", "h_in"]

    @property
    def output_names(self) -> list[str]:
        return ["actions", "h_out", "c_out"] if self.rnn_type == "lstm" else ["actions", "h_out"]
