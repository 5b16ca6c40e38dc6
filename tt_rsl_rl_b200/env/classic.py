"""Seeded batched test environments for learning checks (the reference plugin's harness has the same roles:
``rsl_rl_tt/testing/envs.py``): cart-pole, a partially observed cart-pole (positions only, for recurrent policies), a
cart-pole with a 2-D observation map (for convolutional encoders), pendulum swing-up, and a 12-D trajectory-tracking task with a privileged critic group, terminations, time-outs and
``extras["log"]``. All state lives in device tensors; resets and noise come from a per-environment generator.

Dynamics (standard formulations, written from their physics):

* cart-pole: Barto, Sutton & Anderson (1983) cart-pole with Euler integration (tau = 0.02 s, pole half-length 0.5 m,
  cart 1 kg, pole 0.1 kg), continuous force ``10 N * clip(a, -1, 1)``, termination at |x| > 2.4 m or
  |theta| > 12 degrees, reward 1 per surviving step;
* pendulum: rigid pendulum (m = l = 1, g = 10, dt = 0.05 s), torque ``clip(2 a, -2, 2)``, speed limit 8 rad/s,
  reward ``-(wrap(theta)^2 + 0.1 thetadot^2 + 0.001 u^2)``, no termination;
* tracking: a damped 12-D point mass follows a sinusoidal target per dimension (random amplitude, frequency and phase
  per episode); the actor sees tracking errors and its last action, the critic also the target's parameters.
"""

from __future__ import annotations

import math

import torch

from ..utils.tensordict import TensorDict
from .vec_env import VecEnv


class _SeededBatchEnv(VecEnv):
    num_actions: int = 1
    time_out_steps: int = 500
    step_dt: float = 0.02  # simulated seconds per step (RND scales its weight by it)
    obs_groups_cfg: dict = {"actor": ["policy"], "critic": ["policy"]}

    def __init__(self, num_envs: int, seed: int = 0, device: str | torch.device = "cpu") -> None:
        self.num_envs = num_envs
        self.device = torch.device(device)
        self.max_episode_length = self.time_out_steps
        self.episode_length_buf = torch.zeros(num_envs, dtype=torch.long, device=self.device)
        self.gen = torch.Generator(device=self.device).manual_seed(seed)
        self.cfg = {"env": type(self).__name__, "num_envs": num_envs, "seed": seed,
                    "max_episode_length": self.time_out_steps}
        self._reset(torch.ones(num_envs, dtype=torch.bool, device=self.device))

    @property
    def unwrapped(self):
        return self

    def _uniform(self, *shape, lo: float = 0.0, hi: float = 1.0) -> torch.Tensor:
        return torch.rand(*shape, generator=self.gen, device=self.device) * (hi - lo) + lo

    # subclass hooks
    def _reset(self, mask: torch.Tensor) -> None:
        raise NotImplementedError

    def _advance(self, actions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, dict]:
        """Apply actions; return (rewards [N], terminated [N] bool, log scalars)."""
        raise NotImplementedError

    def _observe(self) -> TensorDict:
        raise NotImplementedError

    def get_observations(self):
        return self._observe()

    def step(self, actions: torch.Tensor):
        rewards, terminated, log = self._advance(actions.to(self.device).float())
        self.episode_length_buf += 1
        time_outs = (self.episode_length_buf >= self.time_out_steps) & ~terminated
        dones = terminated | time_outs
        if bool(dones.any()):
            self._reset(dones)
            self.episode_length_buf[dones] = 0
        extras = {"time_outs": time_outs.float(), "log": log}
        return self._observe(), rewards, dones.float(), extras


class BatchedCartPole(_SeededBatchEnv):
    num_actions = 1
    time_out_steps = 500
    G, M_CART, M_POLE, HALF_LEN, FORCE, TAU = 9.8, 1.0, 0.1, 0.5, 10.0, 0.02
    step_dt = TAU
    X_LIMIT, THETA_LIMIT = 2.4, 12.0 * math.pi / 180.0

    def _reset(self, mask: torch.Tensor) -> None:
        fresh = self._uniform(self.num_envs, 4, lo=-0.05, hi=0.05)
        if not hasattr(self, "s"):
            self.s = fresh
        else:
            self.s[mask] = fresh[mask]

    def _advance(self, actions):
        x, xd, th, thd = self.s.unbind(1)
        force = self.FORCE * actions[:, 0].clamp(-1.0, 1.0)
        total = self.M_CART + self.M_POLE
        pml = self.M_POLE * self.HALF_LEN
        cos, sin = torch.cos(th), torch.sin(th)
        temp = (force + pml * thd * thd * sin) / total
        thacc = (self.G * sin - cos * temp) / (self.HALF_LEN * (4.0 / 3.0 - self.M_POLE * cos * cos / total))
        xacc = temp - pml * thacc * cos / total
        self.s = torch.stack([x + self.TAU * xd, xd + self.TAU * xacc, th + self.TAU * thd, thd + self.TAU * thacc], 1)
        terminated = (self.s[:, 0].abs() > self.X_LIMIT) | (self.s[:, 2].abs() > self.THETA_LIMIT)
        rewards = torch.ones(self.num_envs, device=self.device)
        return rewards, terminated, {"pole_angle": self.s[:, 2].abs().mean()}

    def _observe(self):
        return TensorDict({"policy": self.s.clone()}, batch_size=[self.num_envs], device=self.device)


class BatchedCartPolePO(BatchedCartPole):
    """Cart-pole observing positions only (cart position and pole angle): velocities must be inferred from history."""

    def _observe(self):
        return TensorDict({"policy": self.s[:, [0, 2]].clone()}, batch_size=[self.num_envs], device=self.device)


class BatchedCartPoleImage(BatchedCartPole):
    """Cart-pole with a 2-D observation group for convolutional encoders: ``"image"`` is a 1 x 12 x 12 map holding a
    Gaussian bump at (cart position, pole angle) on a grid spanning the termination limits; ``"policy"`` keeps the
    velocities."""

    GRID = 12
    obs_groups_cfg = {"actor": ["policy", "image"], "critic": ["policy", "image"]}

    def _observe(self):
        g = torch.linspace(-1.0, 1.0, self.GRID, device=self.device)
        px = (self.s[:, 0] / self.X_LIMIT)[:, None, None]
        pt = (self.s[:, 2] / self.THETA_LIMIT)[:, None, None]
        image = torch.exp(-((g[None, :, None] - px) ** 2 + (g[None, None, :] - pt) ** 2) / 0.05)
        return TensorDict({"policy": self.s[:, [1, 3]].clone(), "image": image.unsqueeze(1)},
                          batch_size=[self.num_envs], device=self.device)


class BatchedPendulum(_SeededBatchEnv):
    num_actions = 1
    time_out_steps = 200
    G, MASS, LEN, DT, MAX_SPEED, MAX_TORQUE = 10.0, 1.0, 1.0, 0.05, 8.0, 2.0
    step_dt = DT

    def _reset(self, mask):
        th = self._uniform(self.num_envs, lo=-math.pi, hi=math.pi)
        thd = self._uniform(self.num_envs, lo=-1.0, hi=1.0)
        if not hasattr(self, "th"):
            self.th, self.thd = th, thd
        else:
            self.th[mask], self.thd[mask] = th[mask], thd[mask]

    def _advance(self, actions):
        u = (2.0 * actions[:, 0]).clamp(-self.MAX_TORQUE, self.MAX_TORQUE)
        wrapped = torch.remainder(self.th + math.pi, 2.0 * math.pi) - math.pi
        cost = wrapped.square() + 0.1 * self.thd.square() + 0.001 * u.square()
        acc = 3.0 * self.G / (2.0 * self.LEN) * torch.sin(self.th) + 3.0 / (self.MASS * self.LEN ** 2) * u
        self.thd = (self.thd + acc * self.DT).clamp(-self.MAX_SPEED, self.MAX_SPEED)
        self.th = self.th + self.thd * self.DT
        terminated = torch.zeros(self.num_envs, dtype=torch.bool, device=self.device)
        return -cost, terminated, {"upright": (wrapped.abs() < 0.3).float().mean()}

    def _observe(self):
        obs = torch.stack([torch.cos(self.th), torch.sin(self.th), self.thd], 1)
        return TensorDict({"policy": obs}, batch_size=[self.num_envs], device=self.device)


class Tracking12(_SeededBatchEnv):
    """Damped 12-D point mass tracking a per-dimension sinusoid; privileged critic observations."""

    num_actions = 12
    time_out_steps = 400
    obs_groups_cfg = {"actor": ["policy"], "critic": ["policy", "privileged"]}
    DT, DAMPING, ACC_LIMIT, LOST = 0.05, 0.5, 4.0, 3.0
    step_dt = DT

    def _reset(self, mask):
        N, D = self.num_envs, 12
        fresh = {
            "p": self._uniform(N, D, lo=-0.2, hi=0.2), "v": torch.zeros(N, D, device=self.device),
            "amp": self._uniform(N, D, lo=0.2, hi=1.0), "omega": self._uniform(N, D, lo=0.5, hi=2.0),
            "phase": self._uniform(N, D, lo=0.0, hi=2.0 * math.pi), "t": torch.zeros(N, device=self.device),
            "a_prev": torch.zeros(N, D, device=self.device),
        }
        if not hasattr(self, "p"):
            for k, v in fresh.items():
                setattr(self, k, v)
        else:
            for k, v in fresh.items():
                getattr(self, k)[mask] = v[mask]

    def _target(self):
        arg = self.omega * self.t[:, None] + self.phase
        return self.amp * torch.sin(arg), self.amp * self.omega * torch.cos(arg)

    def _advance(self, actions):
        a = actions.clamp(-self.ACC_LIMIT, self.ACC_LIMIT)
        self.v = self.v + self.DT * (a - self.DAMPING * self.v)
        self.p = self.p + self.DT * self.v
        self.t = self.t + self.DT
        self.a_prev = a
        r, _ = self._target()
        err = (self.p - r).norm(dim=1)
        rewards = 1.0 - err.square() - 0.01 * a.square().sum(dim=1)
        terminated = err > self.LOST
        return rewards, terminated, {"tracking_error": err.mean()}

    def _observe(self):
        r, rd = self._target()
        policy = torch.cat([self.p - r, self.v - rd, self.a_prev], dim=1)
        privileged = torch.cat([r, rd, self.omega, torch.sin(self.phase)], dim=1)
        return TensorDict({"policy": policy, "privileged": privileged}, batch_size=[self.num_envs], device=self.device)


ENV_CLASSES = {"cartpole": BatchedCartPole, "cartpole_po": BatchedCartPolePO, "cartpole_image": BatchedCartPoleImage,
               "pendulum": BatchedPendulum, "tracking12": Tracking12}


def env_class(name: str) -> type[_SeededBatchEnv]:
    """The test environment class registered under ``name`` (a key of :data:`ENV_CLASSES`)."""
    try:
        return ENV_CLASSES[name]
    except KeyError:
        raise KeyError(f"unknown test environment {name!r}; known: {sorted(ENV_CLASSES)}") from None


def make_env(name: str, num_envs: int, seed: int = 0, device: str | torch.device = "cpu") -> _SeededBatchEnv:
    """Build the seeded test environment ``name`` with ``num_envs`` environments on ``device``."""
    return env_class(name)(num_envs, seed=seed, device=device)


__all__ = ["ENV_CLASSES", "BatchedCartPole", "BatchedCartPoleImage", "BatchedCartPolePO", "BatchedPendulum",
           "Tracking12", "env_class", "make_env"]
