"""Mirror functions of the seeded test environments, in the form ``symmetry_cfg["data_augmentation_func"]`` expects:
``func(env, obs, actions)`` with either argument possibly ``None``; the result ``(obs_aug, actions_aug)`` holds the
original rows first and then every mirrored copy (``[R * K, ...]``). A config names them as
``"tt_rsl_rl_b200.testing.symmetry:<name>"``. The reference plugin keeps functions with the same roles for its own test
environments (``rsl_rl_tt/testing/symmetry.py:1-80``); these are derived from the dynamics of
:mod:`tt_rsl_rl_b200.env.classic`:

* cart-pole (full and position-only): every state variable is odd under the reflection x -> -x, theta -> -theta, and
  so is the force (K = 2);
* pendulum: theta -> -theta maps the observation ``[cos, sin, thetadot]`` to ``[cos, -sin, -thetadot]`` and the torque
  to its negative; the cost is even (K = 2);
* tracking12: the dimensions are independent with identically distributed targets, so the sign flip (target phase
  + pi: the reference position and velocity, the tracking errors, the velocities and the actions change sign; the
  frequency does not; ``sin(phase)`` changes sign) and the swap of dimensions ``j <-> j + 6`` are symmetries, as is
  their composition (``tracking12_dihedral_mirror``, K = 4).

Three functions that are NOT signed permutations exercise the probe that turns a mirror function into device maps:
an affine one (constant offset), one that mixes two observation groups, and a nonlinear one that agrees with a signed
permutation on basis vectors.
"""

from __future__ import annotations

import torch

from ..utils.tensordict import TensorDict

_D = 12  # dimensions of Tracking12


def _assemble(obs, actions, obs_maps, act_maps):
    """Concatenate the originals and each copy: ``obs_maps[k]`` maps a dict of group tensors to copy ``k + 1``."""
    out_obs = out_act = None
    if obs is not None:
        groups = {k: obs[k] for k in obs.keys()}
        copies = [groups] + [fn(groups) for fn in obs_maps]
        rows = obs.batch_size[0] * len(copies)
        out_obs = TensorDict({k: torch.cat([c[k] for c in copies], dim=0) for k in groups}, batch_size=[rows],
                             device=obs.device)
    if actions is not None:
        out_act = torch.cat([actions] + [fn(actions) for fn in act_maps], dim=0)
    return out_obs, out_act


def _neg_all(groups):
    return {k: -v for k, v in groups.items()}


def cartpole_mirror(env=None, obs=None, actions=None):
    """Reflection of the cart-pole (position-only variant included): every observation and the force are odd."""
    return _assemble(obs, actions, [_neg_all], [lambda a: -a])


def pendulum_mirror(env=None, obs=None, actions=None):
    """theta -> -theta: ``[cos, sin, thetadot] -> [cos, -sin, -thetadot]``, torque -> -torque."""

    def flip(groups):
        sign = torch.tensor([1.0, -1.0, -1.0], device=groups["policy"].device)
        return {k: v * sign for k, v in groups.items()}

    return _assemble(obs, actions, [flip], [lambda a: -a])


def _swap_halves(x):
    """Swap dimension ``j`` with ``j + 6`` inside every block of 12 features."""
    idx = torch.arange(x.shape[-1], device=x.device).reshape(-1, _D)
    idx = torch.cat([idx[:, _D // 2:], idx[:, : _D // 2]], dim=1).reshape(-1)
    return x[..., idx]


def _flip_tracking(groups):
    # policy = [p - r, v - rd, a_prev]: all odd. privileged = [r, rd, omega, sin(phase)]: r, rd, sin odd; omega even.
    sign = torch.cat([-torch.ones(2 * _D), torch.ones(_D), -torch.ones(_D)]).to(groups["privileged"].device)
    return {"policy": -groups["policy"], "privileged": groups["privileged"] * sign}


def _swap_tracking(groups):
    return {k: _swap_halves(v) for k, v in groups.items()}


def tracking12_sign_mirror(env=None, obs=None, actions=None):
    """Sign flip of every tracked dimension (K = 2)."""
    return _assemble(obs, actions, [_flip_tracking], [lambda a: -a])


def tracking12_dihedral_mirror(env=None, obs=None, actions=None):
    """Identity, sign flip, half swap and their composition (K = 4)."""
    return _assemble(obs, actions,
                     [_flip_tracking, _swap_tracking, lambda g: _flip_tracking(_swap_tracking(g))],
                     [lambda a: -a, _swap_halves, lambda a: -_swap_halves(a)])


# ---- functions the signed-permutation probe must refuse ---------------------------------------------------------------
def tracking12_affine_mirror(env=None, obs=None, actions=None):
    """A sign flip plus a constant offset (affine, not linear)."""
    return _assemble(obs, actions, [lambda g: {k: -v + 0.25 for k, v in g.items()}], [lambda a: -a + 0.5])


def tracking12_mixing_mirror(env=None, obs=None, actions=None):
    """Copy 1 of the privileged group reads the policy group (a map across groups)."""

    def mix(groups):
        priv = groups["privileged"].clone()
        priv[:, :_D] = groups["policy"][:, :_D]
        return {"policy": -groups["policy"], "privileged": priv}

    return _assemble(obs, actions, [mix], [lambda a: -a])


def tracking12_cubic_mirror(env=None, obs=None, actions=None):
    """``x -> -x^3``: equal to the sign flip on 0 / 1 basis vectors, nonlinear elsewhere."""
    return _assemble(obs, actions, [lambda g: {k: -(v ** 3) for k, v in g.items()}], [lambda a: -a])


MIRRORS = {"cartpole": cartpole_mirror, "cartpole_po": cartpole_mirror, "pendulum": pendulum_mirror,
           "tracking12": tracking12_sign_mirror}

__all__ = ["MIRRORS", "cartpole_mirror", "pendulum_mirror", "tracking12_affine_mirror", "tracking12_cubic_mirror",
           "tracking12_dihedral_mirror", "tracking12_mixing_mirror", "tracking12_sign_mirror"]
