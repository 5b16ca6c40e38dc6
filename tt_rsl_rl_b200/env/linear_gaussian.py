"""Seeded synthetic linear-Gaussian environment used by the benchmark configurations.

Dynamics ``s' = A s + B a + noise_std * eps`` with ``eps ~ N(0, I)``; ``A`` (S x S) and ``B`` (S x A) are drawn from a
seed, ``A`` scaled to spectral radius ``rho`` and ``B`` to spectral norm ``rho``. Reward ``-|s'|^2 - 0.01 |a|^2``.
Episodes terminate at random with probability ``reset_prob`` per step (a termination) and are truncated at
``episode_length`` steps (a time-out, reported in ``extras["time_outs"]``); a reset draws ``s ~ N(0, I)``.

Observations: group ``"policy"`` is the state ``s`` (S values); group ``"critic"`` appends ``privileged_dim``
privileged features (|s|^2 / S, |a_prev|^2 / A, episode progress, then zeros) when ``privileged_dim > 0``.

``step`` performs only asynchronous device work (no host synchronisation), so it can be captured in a CUDA graph.

Observation buffers: by default the PyTorch-op step alternates between two observation buffers, because rsl_rl keeps a
reference to the observations a policy acted on and copies them into its storage after the next step. With
``inplace_obs=True`` the observations are rewritten in place every step (the consumer copies them when it acts, as
this framework's engines do); such an environment on CUDA is ``graph_capturable``. Both modes do the same device work.

With ``host_noise=True`` the process noise is read from a pinned host pool and copied to the device every step (the
input of an end-to-end measurement). With ``rollout_steps=T`` on CUDA the copy of step ``k + 1``'s noise runs on a
side stream while step ``k`` computes (double buffer); the first step of every window of ``T`` steps copies in line,
so a window that is captured as one CUDA graph joins every copy it forks. ``T`` must then equal the rollout length.

The same class serves the CPU path, the CUDA path and the unmodified-reference benchmark arm; it depends only on torch
and a TensorDict class. It implements rsl_rl's environment interface (``rsl_rl/env/vec_env.py:14-102``); the
reference plugin benchmarks with a null environment instead (``scripts/bench_matrix.py:34-51``), which this package
also has (``env/null.py``).
"""

from __future__ import annotations

import torch

try:  # the TensorDict class the caller's framework uses (real package or a stand-in on sys.path)
    from tensordict import TensorDict  # type: ignore
except ImportError:  # pragma: no cover - depends on the environment
    from ..utils.tensordict import TensorDict

from .vec_env import VecEnv


def make_system_matrices(state_dim: int, action_dim: int, seed: int, rho: float = 0.95):
    """Seeded ``(A, B)`` on the CPU: A with spectral radius ``rho``, B with largest singular value ``rho``."""
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(state_dim, state_dim, generator=g, dtype=torch.float64)
    radius = torch.linalg.eigvals(A).abs().max().item()
    A = A * (rho / radius)
    B = torch.randn(state_dim, action_dim, generator=g, dtype=torch.float64)
    B = B * (rho / torch.linalg.matrix_norm(B, ord=2).item())
    return A.float(), B.float()


class LinearGaussianVecEnv(VecEnv):
    def __init__(self, num_envs: int, obs_dim: int = 48, num_actions: int = 12, privileged_dim: int = 0,
                 episode_length: int = 1000, reset_prob: float = 0.005, noise_std: float = 0.05, seed: int = 0,
                 device: str | torch.device = "cpu", host_noise: bool = False, host_noise_pool_steps: int = 8,
                 step_dt: float = 0.02, fused: bool | None = None, inplace_obs: bool = False,
                 rollout_steps: int | None = None) -> None:
        self.num_envs = num_envs
        self.num_obs = obs_dim
        self.num_actions = num_actions
        self.privileged_dim = privileged_dim
        self.max_episode_length = episode_length
        self.reset_prob = reset_prob
        self.noise_std = noise_std
        self.device = torch.device(device)
        self.step_dt = step_dt
        self.cfg = {
            "num_envs": num_envs, "obs_dim": obs_dim, "num_actions": num_actions, "privileged_dim": privileged_dim,
            "episode_length": episode_length, "reset_prob": reset_prob, "noise_std": noise_std, "seed": seed,
        }
        A, B = make_system_matrices(obs_dim, num_actions, seed)
        # row-vector form: s'[n] = s[n] @ A^T + a[n] @ B^T
        self.At = A.t().contiguous().to(self.device)
        self.Bt = B.t().contiguous().to(self.device)
        gen = torch.Generator(device="cpu").manual_seed(seed + 1)
        self.state = torch.randn(num_envs, obs_dim, generator=gen).to(self.device)
        self.episode_length_buf = torch.zeros(num_envs, dtype=torch.long, device=self.device)
        self.rewards = torch.zeros(num_envs, device=self.device)
        self.dones = torch.zeros(num_envs, device=self.device)
        self.time_outs = torch.zeros(num_envs, device=self.device)
        self._noise = torch.zeros(num_envs, obs_dim, device=self.device)
        self._reset_noise = torch.zeros(num_envs, obs_dim, device=self.device)
        self._uniform = torch.zeros(num_envs, device=self.device)
        self._next = torch.zeros(num_envs, obs_dim, device=self.device)
        self._policy_obs = torch.zeros(num_envs, obs_dim, device=self.device)
        crit_dim = obs_dim + privileged_dim
        self._critic_obs = torch.zeros(num_envs, crit_dim, device=self.device) if privileged_dim > 0 else None
        self.host_noise = host_noise
        self._copy_stream = None
        if host_noise:
            pin = self.device.type == "cuda"
            pool = torch.randn(host_noise_pool_steps, num_envs, obs_dim, generator=gen)
            self._host_pool = pool.pin_memory() if pin else pool
            self._host_step = 0
            if pin and rollout_steps is not None and rollout_steps > 1:
                # double-buffered prefetch of the next step's noise on a copy stream
                self._prefetch_window = int(rollout_steps)
                self._copy_stream = torch.cuda.Stream(device=self.device)
                self._noise_slots = (self._noise, torch.zeros_like(self._noise))
                self._noise_ready = None
        self._write_obs(torch.zeros(num_envs, num_actions, device=self.device))
        self._obs = self._make_obs_dict()
        # fused device step (the whole transition in one kernel; state width a multiple of 4 up to 128, at most 64
        # actions); None: on CUDA when the framework's extension is available. The PyTorch-op step below is the
        # specification and the CPU path.
        if fused is None:
            fused = (self.device.type == "cuda" and obs_dim % 4 == 0 and obs_dim <= 128 and num_actions <= 64
                     and _extension_available())
        self.fused = bool(fused)
        self.inplace_obs = bool(inplace_obs) and not self.fused
        if not self.fused and not self.inplace_obs:
            # the PyTorch-op step alternates between two observation buffers: the observations a policy acted on stay
            # intact until the algorithm has stored them after the next step (rsl_rl keeps a reference to them)
            self._spare_obs = (torch.zeros_like(self._policy_obs),
                               None if self._critic_obs is None else torch.zeros_like(self._critic_obs))
        if self.fused:
            self._env_counter = torch.zeros(1, dtype=torch.int64, device=self.device)
            self._env_ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._env_seed = (seed * 0x9E3779B97F4A7C15 + 0x5851F42D4C957F2D) % (2**63)

    @property
    def graph_capturable(self) -> bool:
        """The fused step and the in-place PyTorch-op step on CUDA only enqueue device work into fixed buffers, so a
        rollout can be one CUDA graph."""
        return self.fused or (self.inplace_obs and self.device.type == "cuda")

    # ---- VecEnv -----------------------------------------------------------------------------------------------------
    @property
    def unwrapped(self) -> LinearGaussianVecEnv:
        return self

    def get_observations(self):
        return self._obs

    def _make_obs_dict(self):
        groups = {"policy": self._policy_obs}
        if self._critic_obs is not None:
            groups["critic"] = self._critic_obs
        return TensorDict(groups, batch_size=[self.num_envs], device=self.device)

    def _draw_noise(self) -> torch.Tensor:
        """This step's process noise: drawn on the device, or copied from the pinned host pool."""
        if not self.host_noise:
            self._noise.normal_()
            return self._noise
        k = self._host_step
        self._host_step += 1
        pool = self._host_pool
        if self._copy_stream is None:
            self._noise.copy_(pool[k % pool.shape[0]], non_blocking=True)
            return self._noise
        cur = torch.cuda.current_stream(self.device)
        phase = k % self._prefetch_window
        slot = self._noise_slots[k % 2]
        if phase == 0 or self._noise_ready is None:
            slot.copy_(pool[k % pool.shape[0]], non_blocking=True)
        else:
            cur.wait_event(self._noise_ready)  # the copy that step k - 1 started
        self._noise_ready = None
        if phase + 1 < self._prefetch_window:
            # slot (k + 1) % 2 was last read by step k - 1, whose work is already on the current stream
            self._copy_stream.wait_stream(cur)
            with torch.cuda.stream(self._copy_stream):
                self._noise_slots[(k + 1) % 2].copy_(pool[(k + 1) % pool.shape[0]], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(self._copy_stream)
            self._noise_ready = ready
        return slot

    def _write_obs(self, actions: torch.Tensor) -> None:
        self._policy_obs.copy_(self.state)
        if self._critic_obs is not None:
            S, A = self.num_obs, self.num_actions
            self._critic_obs[:, :S].copy_(self.state)
            extra = self._critic_obs[:, S:]
            extra.zero_()
            extra[:, 0].copy_(self.state.square().sum(dim=1) / S)
            if self.privileged_dim > 1:
                extra[:, 1].copy_(actions.square().sum(dim=1) / A)
            if self.privileged_dim > 2:
                extra[:, 2].copy_(self.episode_length_buf.float() / float(self.max_episode_length))

    def step(self, actions: torch.Tensor):
        a = actions.to(self.device)
        if self.fused:
            return self._fused_step(a)
        noise = self._draw_noise()
        # s' = A s + B a + sigma * eps
        torch.addmm(torch.mm(self.state, self.At), a, self.Bt, out=self._next)
        self._next.add_(noise, alpha=self.noise_std)
        # reward on the new state and the applied action
        torch.sum(self._next.square(), dim=1, out=self.rewards)
        self.rewards.add_(a.square().sum(dim=1), alpha=0.01).neg_()
        # episode bookkeeping: random terminations and time-outs
        self.episode_length_buf.add_(1)
        self._uniform.uniform_()
        terminated = self._uniform < self.reset_prob
        timed_out = self.episode_length_buf >= self.max_episode_length
        done = terminated | timed_out
        self.time_outs.copy_(timed_out & ~terminated)
        self.dones.copy_(done)
        # reset finished environments to s ~ N(0, I)
        self._reset_noise.normal_()
        self.state.copy_(torch.where(done.unsqueeze(1), self._reset_noise, self._next))
        self.episode_length_buf.masked_fill_(done, 0)
        if not self.inplace_obs:
            spare = self._spare_obs
            self._spare_obs = (self._policy_obs, self._critic_obs)
            self._policy_obs, self._critic_obs = spare
            self._obs = self._make_obs_dict()
        self._write_obs(a)
        extras = {"time_outs": self.time_outs, "log": {"/state_norm": self.rewards}}
        return self._obs, self.rewards, self.dones, extras


    def _fused_step(self, a: torch.Tensor):
        """Same transition in one kernel of this framework: the matrix-vector products with A and B from shared
        memory, Philox noise, reward, resets and observation writes."""
        noise = self._draw_noise() if self.host_noise else None
        from ..ops import ext

        a = a if a.stride(1) == 1 else a.contiguous()
        ext().lg_env_step(self.At, self.Bt, self.state, a, noise, self.noise_std, self.reset_prob,
                                int(self.max_episode_length), self.episode_length_buf, self.rewards, self.dones,
                                self.time_outs, self._policy_obs, self._critic_obs, self.privileged_dim,
                                self._env_seed, self._env_counter, self._env_ticket)
        extras = {"time_outs": self.time_outs, "log": {"/state_norm": self.rewards}}
        return self._obs, self.rewards, self.dones, extras


def _extension_available() -> bool:
    try:
        from ..ops import ext

        ext()
        return True
    except Exception:  # pragma: no cover - depends on the build
        return False


def humanoid_like(num_envs: int, device: str | torch.device = "cpu", seed: int = 0, **kw) -> LinearGaussianVecEnv:
    """The benchmark shape: actor obs 96, critic obs 99 (3 privileged features), 29 actions."""
    return LinearGaussianVecEnv(num_envs, obs_dim=96, num_actions=29, privileged_dim=3, seed=seed, device=device, **kw)


def spectral_radius(matrix: torch.Tensor) -> float:
    """Largest eigenvalue modulus (used by tests)."""
    return float(torch.linalg.eigvals(matrix.double()).abs().max())


__all__ = ["LinearGaussianVecEnv", "humanoid_like", "make_system_matrices", "spectral_radius"]
