"""Running observation / reward normalisers with the buffers of ``rsl_rl/modules/normalization.py``.

Buffers: ``_mean``, ``_var``, ``_std`` (shape ``[1, *shape]``) and ``count`` (int64), so checkpoints interoperate.
Under ``torch.distributed`` the statistics are global: counts and first/second moments are combined across ranks
around the global mean (``normalization.py:62-71``). The CUDA training path performs the same update in
``ops/csrc/rl_kernels.cu`` (column moments) and the communicator (cross-rank combine).
"""

from __future__ import annotations

import torch
from torch import nn


class EmpiricalNormalization(nn.Module):
    """``y = (x - mean) / (std + eps)`` with running statistics updated by :meth:`update`."""

    def __init__(self, shape: int | tuple[int, ...] | list[int], eps: float = 1e-2, until: int | None = None) -> None:
        super().__init__()
        self.eps = eps
        self.until = until
        self.register_buffer("_mean", torch.zeros(shape).unsqueeze(0))
        self.register_buffer("_var", torch.ones(shape).unsqueeze(0))
        self.register_buffer("_std", torch.ones(shape).unsqueeze(0))
        self.register_buffer("count", torch.tensor(0, dtype=torch.long))

    @property
    def mean(self) -> torch.Tensor:
        return self._mean.squeeze(0).clone()

    @property
    def std(self) -> torch.Tensor:
        return self._std.squeeze(0).clone()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return (x - self._mean) / (self._std + self.eps)

    @torch.jit.unused
    def update(self, x: torch.Tensor) -> None:
        """Fold a batch ``x [B, *shape]`` into the running statistics (no-op in eval mode or after ``until``)."""
        if not self.training:
            return
        if self.until is not None and self.count >= self.until:
            return
        n = torch.tensor(x.shape[0], dtype=self.count.dtype, device=self.count.device)
        batch_mean = x.mean(dim=0, keepdim=True)
        batch_var = x.var(dim=0, unbiased=False, keepdim=True)
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            n, batch_mean, batch_var = combine_moments_distributed(n, batch_mean, batch_var, x.shape[0])
        self.apply_moments(n, batch_mean, batch_var)

    @torch.jit.unused
    def apply_moments(self, n: torch.Tensor, batch_mean: torch.Tensor, batch_var: torch.Tensor) -> None:
        """Running update from a batch of ``n`` samples with the given mean and (biased) variance."""
        self.count += n
        rate = n / self.count
        delta = batch_mean - self._mean
        self._mean += rate * delta
        self._var += rate * (batch_var - self._var + delta * (batch_mean - self._mean))
        # in place: an update inside inference mode (the RND reward normaliser runs in the rollout) keeps the buffer
        # a normal tensor, so a later load_state_dict can still write it
        self._std.copy_(torch.sqrt(self._var))

    @torch.jit.unused
    def inverse(self, y: torch.Tensor) -> torch.Tensor:
        return y * (self._std + self.eps) + self._mean


def combine_moments_distributed(n: torch.Tensor, mean: torch.Tensor, var: torch.Tensor, local_rows: int):
    """Global count, mean and biased variance from per-rank moments (three all-reduces, as upstream)."""
    local_mean = mean
    torch.distributed.all_reduce(n)
    total = mean * local_rows
    torch.distributed.all_reduce(total)
    gmean = total / n
    spread = local_rows * (var + (local_mean - gmean).square())
    torch.distributed.all_reduce(spread)
    return n, gmean, spread / n


class EmpiricalDiscountedVariationNormalization(nn.Module):
    """Divide rewards by the running std of their discounted sum (``normalization.py:86-119``)."""

    def __init__(self, shape: int | tuple[int, ...] | list[int], eps: float = 1e-2, gamma: float = 0.99,
                 until: int | None = None) -> None:
        super().__init__()
        self.emp_norm = EmpiricalNormalization(shape, eps, until)
        self.disc_avg = _DiscountedAverage(gamma)

    def forward(self, rew: torch.Tensor) -> torch.Tensor:
        if self.training:
            self.emp_norm.update(self.disc_avg.update(rew))
        std = self.emp_norm._std
        return rew / std if std > 0 else rew


class _DiscountedAverage:
    """``avg_t = gamma * avg_{t-1} + r_t`` starting from the first reward."""

    def __init__(self, gamma: float) -> None:
        self.avg: torch.Tensor | None = None
        self.gamma = gamma

    def update(self, rew: torch.Tensor) -> torch.Tensor:
        self.avg = rew.clone() if self.avg is None else self.avg * self.gamma + rew
        return self.avg
