"""Recurrent encoder (GRU or LSTM) with an internal hidden state (``rsl_rl/modules/rnn.py``).

Two modes: rollout mode (no masks) runs one time step and keeps the hidden state; batch mode (masks given) runs the
padded trajectories of a recurrent minibatch from the supplied initial hidden state and unpads the output.
Parameter names (``rnn.weight_ih_l0`` ...) are those of ``torch.nn.GRU/LSTM``, as in rsl_rl checkpoints.
"""

from __future__ import annotations

from typing import Union

import torch
import torch.nn as nn

from ..utils.utils import unpad_trajectories

HiddenState = Union[torch.Tensor, tuple[torch.Tensor, torch.Tensor], None]
"""GRU: one tensor ``[layers, N, H]``; LSTM: a ``(h, c)`` pair; ``None`` before the first step."""


class RNN(nn.Module):
    def __init__(self, input_size: int, hidden_dim: int = 256, num_layers: int = 1, type: str = "lstm") -> None:
        super().__init__()
        cls = nn.GRU if type.lower() == "gru" else nn.LSTM
        self.rnn = cls(input_size=input_size, hidden_size=hidden_dim, num_layers=num_layers)
        self.hidden_state: HiddenState = None

    @property
    def is_lstm(self) -> bool:
        return isinstance(self.rnn, nn.LSTM)

    def forward(self, input: torch.Tensor, masks: torch.Tensor | None = None,
                hidden_state: HiddenState = None) -> torch.Tensor:
        if masks is not None:
            if hidden_state is None:
                raise ValueError("Hidden states not passed to RNN module during policy update")
            out, _ = self.rnn(input, hidden_state)
            return unpad_trajectories(out, masks)
        out, self.hidden_state = self.rnn(input.unsqueeze(0), self.hidden_state)
        return out

    def reset(self, dones: torch.Tensor | None = None, hidden_state: HiddenState = None) -> None:
        """Replace the whole state (``dones is None``) or zero the rows of environments that are done."""
        if dones is None:
            self.hidden_state = hidden_state
            return
        if self.hidden_state is None:
            return
        if hidden_state is not None:
            raise NotImplementedError(
                "Resetting the hidden state of done environments with a custom hidden state is not implemented"
            )
        states = self.hidden_state if isinstance(self.hidden_state, tuple) else (self.hidden_state,)
        for s in states:
            s[..., dones == 1, :] = 0.0

    def detach_hidden_state(self, dones: torch.Tensor | None = None) -> None:
        """Cut the autograd graph of the hidden state (all rows, or the rows of done environments)."""
        if self.hidden_state is None:
            return
        if dones is None:
            if isinstance(self.hidden_state, tuple):
                self.hidden_state = tuple(s.detach() for s in self.hidden_state)
            else:
                self.hidden_state = self.hidden_state.detach()
            return
        states = self.hidden_state if isinstance(self.hidden_state, tuple) else (self.hidden_state,)
        for s in states:
            s[..., dones == 1, :] = s[..., dones == 1, :].detach()
