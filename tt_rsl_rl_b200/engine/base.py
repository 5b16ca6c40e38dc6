"""Pieces shared by the fused engines: normaliser views, CUDA-graph capture, device status checks, the observation
normaliser update (local or over the peer exchange) and the captured rollout of graph-capturable environments.

The rollout step replaces ``PPO.act`` / ``process_env_step`` (``rsl_rl/algorithms/ppo.py:124-164``); the normaliser
update is ``EmpiricalNormalization.update`` with its distributed combine (``rsl_rl/modules/normalization.py:51-78``);
capture-once / replay plays the role of the reference plugin's trace mixin (``rsl_rl_tt/traced.py:15-47``) with CUDA
graphs."""

from __future__ import annotations

import torch
import torch.nn as nn

from ..modules import EmpiricalNormalization
from ..ops import ext
from ..utils.timer import HostTransfers


def elu_mlp_reason(model) -> str | None:
    """None if ``model.mlp`` is a Linear/ELU(alpha=1) stack the fused GEMM epilogues cover, else the reason."""
    return elu_stack_reason(getattr(model, "mlp", None))


def elu_stack_reason(mlp) -> str | None:
    """None if the sequential ``mlp`` holds only Linear, ELU(alpha=1) and Unflatten layers, else the reason."""
    if mlp is None:
        return "model has no MLP head"
    for m in mlp:
        if isinstance(m, nn.Linear) or isinstance(m, nn.Unflatten):
            continue
        if not isinstance(m, nn.ELU) or m.alpha != 1.0:
            return f"activation {type(m).__name__} is not fused (ELU only)"
    return None


class EngineBase:
    device: torch.device
    status: torch.Tensor
    nonfinite: torch.Tensor
    comm = None
    use_graphs: bool
    T: int

    def _init_base(self) -> None:
        self._rollout_graph = None
        self._rollout_calls = 0
        self._rollout_obs = None
        self._rollout_delta = None

    # ---- normaliser views --------------------------------------------------------------------------------------------
    @staticmethod
    def _norm_tensors(model):
        return EngineBase._norm_views(model.obs_normalizer)

    @staticmethod
    def _norm_views(norm):
        if isinstance(norm, EmpiricalNormalization):
            return norm._mean.view(-1), norm._std.view(-1), norm.eps
        return None, None, 0.0

    @staticmethod
    def _group_tensors(obs, groups):
        return [obs[g] if obs[g].is_contiguous() else obs[g].contiguous() for g in groups]

    def _alloc_norm_scratch(self, name: str, rows: int, D: int) -> None:
        dev = self.device
        if not hasattr(self, "colstats_partial"):
            self.colstats_partial, self.moments_local, self.moments_global = {}, {}, {}
        if not hasattr(self, "stats_chunks"):
            self.stats_chunks = {}
        self.stats_chunks[name] = ext().colstats_chunks(rows)
        self.colstats_partial[name] = torch.zeros(2 * self.stats_chunks[name] * D, dtype=torch.float64, device=dev)
        self.moments_local[name] = torch.zeros(2 + 2 * D, dtype=torch.float64, device=dev)
        self.moments_global[name] = torch.zeros_like(self.moments_local[name])

    def _normalizer_update(self, name: str, model, obs: torch.Tensor, rows: int, D: int) -> None:
        """Running-moment update of ``model``'s normaliser from ``obs[:rows, :D]`` (global over ranks when
        data-parallel: per-rank column sums, rank-ordered peer all-reduce, then the running update)."""
        self._norm_module_update(name, model.obs_normalizer, model.obs_normalization, obs, rows, D)

    def _norm_module_update(self, name: str, norm, enabled: bool, obs: torch.Tensor, rows: int, D: int) -> None:
        if not isinstance(norm, EmpiricalNormalization) or not enabled or not norm.training:
            return
        C = ext()
        partial = self.colstats_partial[name]
        C.colstats(obs, rows, obs.stride(0), D, partial)
        until = -1 if norm.until is None else int(norm.until)
        mean, var, std = norm._mean.view(-1), norm._var.view(-1), norm._std.view(-1)
        chunks = self.stats_chunks[name]
        if self.comm is None:
            C.norm_update(partial, chunks, rows, D, mean, var, std, norm.count, until, None, False)
            return
        local, glob = self.moments_local[name], self.moments_global[name]
        C.norm_update(partial, chunks, rows, D, mean, var, std, norm.count, until, local, True)
        self.comm.allreduce_f64(local, glob, self.status)
        C.norm_update(glob[2:], 1, rows * self.world, D, mean, var, std, norm.count, until, None, False)

    # ---- actor / critic concurrency ----------------------------------------------------------------------------------
    def _init_streams(self, b200_cfg: dict) -> None:
        """A second stream for the model whose work is independent of the other's (``b200_cfg.model_streams`` = 2)."""
        self._side = torch.cuda.Stream(device=self.device) if int(b200_cfg.get("model_streams", 2)) > 1 else None

    def _in_parallel(self, main_fn, side_fn) -> None:
        """Run ``side_fn`` on the side stream and ``main_fn`` on the current stream, both ordered after the work
        enqueued so far and joined before anything enqueued afterwards (a fork / join in a captured graph)."""
        side = getattr(self, "_side", None)
        if side is None:
            main_fn()
            side_fn()
            return
        cur = torch.cuda.current_stream(self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            side_fn()
        main_fn()
        cur.wait_stream(side)

    # ---- graphs and status --------------------------------------------------------------------------------------------
    def _capture(self, fn):
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

    def _check_status(self) -> None:
        st = HostTransfers.read(self.status, "status")
        if st[0] != 0:
            self.status.zero_()
            if st[0] == 8:  # kBadIndex, reported by builds with -DRL_DEBUG_BOUNDS
                raise IndexError(f"a kernel read an index outside its tensor: site={st[1]} block={st[2]} "
                                 f"count={st[3]} (the access was redirected to index 0)")
            from ..parallel import CommTimeoutError

            raise CommTimeoutError(f"device status error code={st[0]} site={st[1]} block={st[2]} count={st[3]}")

    def check_finite(self, obs, rewards) -> None:
        """Non-finite rewards are flagged on the device by ``process_step``; nothing to do per step."""

    def raise_if_nonfinite(self) -> None:
        if int(HostTransfers.read(self.nonfinite, "nonfinite")[0]) != 0:
            self.nonfinite.zero_()
            raise ValueError("The rewards returned by the environment contain NaN or Inf values.")

    # ---- captured rollout (graph-capturable environments) -------------------------------------------------------------
    def can_capture_rollout(self, env, cfg) -> bool:
        """A rollout can be one CUDA graph when the environment only enqueues device work (``graph_capturable``)."""
        return self.use_graphs and bool(getattr(env, "graph_capturable", False))

    def _rollout_steps(self, env, logger, cfg):
        obs = env.get_observations()
        for _ in range(self.T):
            actions = self.act(obs)
            obs, rewards, dones, extras = env.step(actions)
            self.process_env_step(obs, rewards, dones, extras)
            logger.process_env_step(rewards, dones, extras, getattr(self, "intrinsic_for_logger", None))
        return obs

    def run_captured_rollout(self, env, logger, cfg):
        """Run ``T`` x (act, env step, store, episode bookkeeping); from the second call on as one graph replay.

        The graph replays exactly the captured work: the environment must keep returning the same observation,
        reward and done tensors (updated in place), as ``graph_capturable`` environments do. Host-side counters of
        the logger are advanced by the captured amount after each replay.
        """
        if self._rollout_calls == 0:
            obs = self._rollout_steps(env, logger, cfg)
        else:
            if self._rollout_graph is None:
                before = logger.host_state()
                t0 = self.t
                holder = {}
                self._rollout_graph = self._capture(lambda: holder.setdefault("obs", self._rollout_steps(env, logger,
                                                                                                         cfg)))
                self._rollout_obs = holder["obs"]
                self._rollout_delta = (before, logger.host_state())
                logger.set_host_state(before)
                self.t = t0
            self._before_replay()
            self._rollout_graph.replay()
            logger.advance_host_state(*self._rollout_delta)
            self.t += self.T
            obs = self._rollout_obs
        self._rollout_calls += 1
        if cfg.get("check_for_nan", True):
            self.raise_if_nonfinite()
        return obs

    def _before_replay(self) -> None:
        """Host-side preparation of a replayed rollout (e.g. per-step schedules written to device buffers)."""

    # overridden by the engines
    def act(self, obs):  # pragma: no cover - abstract
        raise NotImplementedError

    def process_env_step(self, obs, rewards, dones, extras) -> None:  # pragma: no cover - abstract
        raise NotImplementedError
