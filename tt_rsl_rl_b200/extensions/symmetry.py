"""Symmetry augmentation and mirror loss (``rsl_rl/extensions/symmetry.py``).

The user supplies ``data_augmentation_func(env, obs, actions) -> (obs_aug, actions_aug)`` returning the original
samples followed by their mirrored copies. On CUDA, :meth:`Symmetry.probe_signed_permutations` evaluates that function
once on basis inputs; when it is a signed permutation per copy (the common case for robot mirror symmetry) the engine
applies it with the gather kernel instead of calling Python every minibatch.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.nn as nn

from ..utils.tensordict import TensorDict
from ..utils.utils import resolve_callable


class Symmetry:
    def __init__(self, env, data_augmentation_func: str | Callable, use_data_augmentation: bool = False,
                 use_mirror_loss: bool = False, mirror_loss_coeff: float = 0.0) -> None:
        self.env = env
        self.use_data_augmentation = use_data_augmentation
        self.use_mirror_loss = use_mirror_loss
        self.mirror_loss_coeff = mirror_loss_coeff
        self.data_augmentation_func = resolve_callable(data_augmentation_func)
        if not (use_data_augmentation or use_mirror_loss):
            print("Symmetry not used for learning. We will use it for logging instead.")

    def augment_batch(self, batch, original_batch_size: int) -> None:
        """Append mirrored observations/actions to the batch and repeat the other rollout fields to match."""
        if not self.use_data_augmentation:
            return
        batch.observations, batch.actions = self.data_augmentation_func(
            env=self.env, obs=batch.observations, actions=batch.actions
        )
        copies = int(batch.observations.batch_size[0] / original_batch_size)
        batch.old_actions_log_prob = batch.old_actions_log_prob.repeat(copies, 1)
        batch.values = batch.values.repeat(copies, 1)
        batch.advantages = batch.advantages.repeat(copies, 1)
        batch.returns = batch.returns.repeat(copies, 1)

    def compute_loss(self, actor: nn.Module, batch, original_batch_size: int) -> torch.Tensor:
        """MSE between the actor mean on mirrored observations and the mirrored actor mean on the originals."""
        if not self.use_data_augmentation:
            batch.observations, _ = self.data_augmentation_func(env=self.env, obs=batch.observations, actions=None)
        means = actor(batch.observations.detach().clone())
        _, mirrored = self.data_augmentation_func(env=self.env, obs=None, actions=means[:original_batch_size])
        loss = nn.functional.mse_loss(means[original_batch_size:], mirrored.detach()[original_batch_size:])
        return loss if self.use_mirror_loss else loss.detach()

    # ---- probing for the CUDA path -------------------------------------------------------------------------------------
    def probe_signed_permutations(self, obs_template, num_actions: int):
        """Express the augmentation as per-copy signed permutations, or return ``None`` if it is not one.

        Returns ``(obs_maps, action_maps)``: ``obs_maps[group] = (perm [K, D] int64, sign [K, D] float)`` such that copy
        k of observation group ``group`` is ``x[:, perm[k]] * sign[k]``; ``action_maps`` likewise for actions. Copy 0
        must be the identity.
        """
        device = next(iter(obs_template.values())).device
        groups = list(obs_template.keys())
        dims = {g: obs_template[g].shape[-1] for g in groups}
        obs_maps = {}
        for g in groups:
            D = dims[g]
            basis = {h: torch.eye(D, device=device) if h == g else torch.zeros(D, dims[h], device=device)
                     for h in groups}
            td = TensorDict(basis, batch_size=[D], device=device)
            out, _ = self.data_augmentation_func(env=self.env, obs=td, actions=None)
            m = out[g]
            K = m.shape[0] // D
            maps = _signed_perm_from_images(m.view(K, D, D))
            if maps is None:
                return None
            obs_maps[g] = maps
        eye_a = torch.eye(num_actions, device=device)
        _, a_out = self.data_augmentation_func(env=self.env, obs=None, actions=eye_a)
        K = a_out.shape[0] // num_actions
        action_maps = _signed_perm_from_images(a_out.view(K, num_actions, num_actions))
        if action_maps is None:
            return None
        if any(perm.shape[0] != K for perm, _ in obs_maps.values()):
            return None  # every group and the actions must have the same number of copies
        if not self._maps_reproduce(obs_template, num_actions, obs_maps, action_maps):
            return None
        return obs_maps, action_maps

    def _maps_reproduce(self, obs_template, num_actions: int, obs_maps: dict, action_maps, rows: int = 5) -> bool:
        """Check the derived maps against the function on random inputs of every group at once.

        Basis vectors alone cannot see a map that reads another group (each group is probed with the others at zero)
        or a nonlinear map that agrees with a signed permutation on 0/1 inputs (``x -> -x**3``)."""
        device = next(iter(obs_template.values())).device
        gen = torch.Generator().manual_seed(0x5EED)
        x = {g: torch.randn(rows, obs_template[g].shape[-1], generator=gen).to(device) for g in obs_template.keys()}
        a = torch.randn(rows, num_actions, generator=gen).to(device)
        out_obs, out_act = self.data_augmentation_func(env=self.env, obs=TensorDict(x, batch_size=[rows], device=device),
                                                       actions=a)

        def matches(got, src, perm, sign):
            want = torch.cat([src[:, perm[k]] * sign[k] for k in range(perm.shape[0])], dim=0)
            return got is not None and got.shape == want.shape and bool(
                torch.allclose(got.float(), want, rtol=1e-3, atol=1e-5))

        if out_obs is None or not all(matches(out_obs[g], x[g], *obs_maps[g]) for g in obs_maps):
            return False
        return matches(out_act, a, *action_maps)


def _signed_perm_from_images(images: torch.Tensor):
    """``images[k, i, :]`` is copy k applied to basis vector i. Returns (perm, sign) with y[j] = sign[j] * x[perm[j]]."""
    K, D, _ = images.shape
    perm = torch.empty(K, D, dtype=torch.long, device=images.device)
    sign = torch.empty(K, D, device=images.device)
    for k in range(K):
        m = images[k]  # m[i, j]: output feature j for input basis i
        nz = m.abs() > 1e-6
        if not bool((nz.sum(0) == 1).all()) or not bool((nz.sum(1) == 1).all()):
            return None
        src = nz.float().argmax(0)
        val = m[src, torch.arange(D, device=m.device)]
        if not bool(((val.abs() - 1).abs() < 1e-5).all()):
            return None
        perm[k] = src
        sign[k] = val.sign()
    return perm, sign


def resolve_symmetry_config(alg_cfg: dict, env) -> dict:
    """Attach the environment to ``symmetry_cfg`` (the augmentation function receives it)."""
    if alg_cfg.get("symmetry_cfg") is not None:
        alg_cfg["symmetry_cfg"]["env"] = env
    else:
        alg_cfg["symmetry_cfg"] = None
    return alg_cfg
