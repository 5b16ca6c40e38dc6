"""Running normalisers of observations and rewards.

Public interface of rsl_rl's ``EmpiricalNormalization`` and ``EmpiricalDiscountedVariationNormalization``
(``rsl_rl/modules/normalization.py``): the buffers ``_mean``, ``_var``, ``_std`` (shape ``[1, *shape]``) and
``count`` (int64), which are checkpoint entries, ``eps`` added to the std in ``forward``, and ``until``.

Design of this package: an update is a merge of :class:`Moments` (count, mean, biased variance). The moments of a
batch are taken locally, made global over the ranks of a ``torch.distributed`` group when one exists (total count,
then the pooled mean, then the pooled spread around it: three all-reduces), and merged into the running moments with
the parallel-variance update (Chan, Golub & LeVeque, 1979), in the operation order rsl_rl uses so that the buffers
agree with it bit for bit. The fused CUDA engines perform the same three steps on the device (column-moment kernel,
peer all-reduce, update kernel).
"""

from __future__ import annotations

from typing import NamedTuple

import torch
from torch import nn


class Moments(NamedTuple):
    """Sample count (int64 tensor), mean and biased variance (``[1, *shape]``) of a set of rows."""

    count: torch.Tensor
    mean: torch.Tensor
    var: torch.Tensor

    @staticmethod
    def of(x: torch.Tensor, count_like: torch.Tensor) -> "Moments":
        n = torch.tensor(x.shape[0], dtype=count_like.dtype, device=count_like.device)
        return Moments(n, x.mean(dim=0, keepdim=True), x.var(dim=0, unbiased=False, keepdim=True))

    def pooled(self, local_rows: int) -> "Moments":
        """The moments of the union of every rank's rows (all ranks call this with their own batch)."""
        n = self.count.clone()
        torch.distributed.all_reduce(n)
        total = self.mean * local_rows
        torch.distributed.all_reduce(total)
        mean = total / n
        spread = local_rows * (self.var + (self.mean - mean).square())
        torch.distributed.all_reduce(spread)
        return Moments(n, mean, spread / n)


class EmpiricalNormalization(nn.Module):
    """``y = (x - mean) / (std + eps)`` with running moments of every batch passed to :meth:`update`."""

    def __init__(self, shape: int | tuple[int, ...] | list[int], eps: float = 1e-2, until: int | None = None) -> None:
        super().__init__()
        self.eps = eps
        self.until = until  # stop learning once this many samples have been seen
        for name, init in (("_mean", torch.zeros), ("_var", torch.ones), ("_std", torch.ones)):
            self.register_buffer(name, init(shape).unsqueeze(0))
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
    def inverse(self, y: torch.Tensor) -> torch.Tensor:
        return y * (self._std + self.eps) + self._mean

    @torch.jit.unused
    def learning(self) -> bool:
        """Whether :meth:`update` changes the statistics (training mode, ``until`` not reached)."""
        return self.training and (self.until is None or bool(self.count < self.until))

    @torch.jit.unused
    def update(self, x: torch.Tensor) -> None:
        """Fold the rows of ``x [B, *shape]`` into the running statistics (global over ranks when distributed)."""
        if not self.learning():
            return
        batch = Moments.of(x, self.count)
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            batch = batch.pooled(x.shape[0])
        self.merge(batch)

    @torch.jit.unused
    def merge(self, batch: Moments) -> None:
        """Parallel-variance merge of ``batch`` into the running moments."""
        self.count += batch.count
        weight = batch.count / self.count
        shift = batch.mean - self._mean
        self._mean += weight * shift
        self._var += weight * (batch.var - self._var + shift * (batch.mean - self._mean))
        # written in place: the RND reward normaliser updates inside the rollout's inference mode, and an inference
        # tensor assigned here could not be overwritten by a later load_state_dict
        self._std.copy_(torch.sqrt(self._var))


class DiscountedSum:
    """Per-environment discounted running sum of rewards, ``s_t = gamma * s_{t-1} + r_t`` (``s_0 = r_0``)."""

    def __init__(self, gamma: float) -> None:
        self.gamma = gamma
        self.avg: torch.Tensor | None = None

    def update(self, rew: torch.Tensor) -> torch.Tensor:
        self.avg = rew.clone() if self.avg is None else self.avg * self.gamma + rew
        return self.avg


class EmpiricalDiscountedVariationNormalization(nn.Module):
    """Reward scaling by the running std of the discounted reward sum (the return scale): rewards of a
    non-stationary source keep a steady magnitude for the value function."""

    def __init__(self, shape: int | tuple[int, ...] | list[int], eps: float = 1e-2, gamma: float = 0.99,
                 until: int | None = None) -> None:
        super().__init__()
        self.emp_norm = EmpiricalNormalization(shape, eps, until)
        self.disc_avg = DiscountedSum(gamma)

    def forward(self, rew: torch.Tensor) -> torch.Tensor:
        if self.training:
            self.emp_norm.update(self.disc_avg.update(rew))
        scale = self.emp_norm._std
        return rew / scale if scale > 0 else rew
