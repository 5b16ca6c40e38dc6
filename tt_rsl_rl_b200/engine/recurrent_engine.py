"""Fused CUDA engine of recurrent PPO (:class:`tt_rsl_rl_b200.models.RNNModel` actor and critic, GRU or LSTM).

Semantics follow upstream's recurrent path (``rsl_rl/storage/rollout_storage.py`` ``recurrent_mini_batch_generator``
and ``rsl_rl/algorithms/ppo.py``): minibatches are contiguous ranges of environments over the whole rollout, in the
same order every epoch; each environment's trajectories are split at dones and re-run from the hidden state stored at
their start. Running the recurrence over the full rollout with the input state masked by ``1 - done`` after every
done is the same computation (a trajectory that starts after a done starts from the reset, zero state; the first one
starts from the state stored at the rollout's first step), and the loss averages over all ``T x envs`` entries as the
unpadded upstream outputs do. That form needs no data-dependent padding, so a minibatch is:

* forward: one GEMM ``gi = x W_ih^T + b_ih`` over all ``T x B`` rows (env-major ``[B, T, .]`` layout, so an env range
  is contiguous), then per step ``gh = h W_hh^T + b_hh`` (tcgen05 GEMM) and the cell (gates, new state, masked
  next-step input, saved activations) -- as one launch with the cell in the GEMM's epilogue when
  ``b200_cfg.rnn_fused_step`` selects it (GRU by default); the MLP head and the PPO loss over all rows;
* backward: head backward including the gradient of its input, then backpropagation through time, per step in
  reverse: the backward cell (gate gradients, bias-gradient column sums, masked recurrent gradients) and the GEMM
  ``dh = dgh W_hh``; the weight gradients of ``W_ih`` and ``W_hh`` as two split-K GEMMs over all rows;
* the gradient reduction and the fused clip + adaptive-LR + Adam kernel shared with the MLP engine.

Rollout steps run the same cell on the persistent per-environment state; ``process_env_step`` masks it at dones.
With RND the intrinsic reward is added during the rollout and the predictor trains on each minibatch as upstream's
does on the padded trajectories (``rnd_part.py``; ``_rnd_minibatch``). The sequence functions also serve the
recurrent distillation student (time-major windows of steps over all environments).
"""

from __future__ import annotations

from itertools import chain

import torch
import torch.nn as nn

from ..modules import GaussianDistribution, HeteroscedasticGaussianDistribution
from ..ops import ext
from ..ops import gemm as G
from ..utils.timer import HostTransfers
from .base import EngineBase, elu_mlp_reason
from .mlp_plan import MLPPlan, pad8, wgrad_splits
from .rnd_part import RndPart, rnd_reason

_TAIL = 5  # exchanged statistics after the parameters: surrogate, value, entropy, kl, (unused)
_GROUP_RND = 2


def _view_from(t: torch.Tensor, offset: int) -> torch.Tensor:
    """1-D view of ``t``'s storage starting ``offset`` elements after its first element (a strided row base)."""
    return t.view(-1)[offset:]


def rnn_model_reason(name: str, m) -> str | None:
    """None if ``m`` is an RNNModel the fused recurrent kernels cover (one unidirectional GRU / LSTM layer with
    biases, hidden size a multiple of 32 up to 1024, a Linear / ELU head), else the reason."""
    from ..models import RNNModel

    if type(m) is not RNNModel:
        return f"{name} type {type(m).__name__} is not the recurrent model"
    rnn = m.rnn.rnn
    if not isinstance(rnn, (nn.GRU, nn.LSTM)):
        return f"{name} recurrent layer {type(rnn).__name__}"
    if rnn.num_layers != 1 or not rnn.bias or rnn.bidirectional or getattr(rnn, "proj_size", 0):
        return f"{name}: only single-layer, unidirectional RNNs with biases are fused"
    if rnn.hidden_size % 32 or rnn.hidden_size > 1024:
        return f"{name}: hidden size must be a multiple of 32 up to 1024"
    reason = elu_mlp_reason(m)
    if reason:
        return f"{name}: {reason}"
    if m.obs_dim > 1024:
        return f"{name} observation width {m.obs_dim} too large"
    return None


class _RecurrentNet:
    """Device plan of one RNNModel: bf16 weight shadows, rollout state, env-major minibatch buffers, the MLP head."""

    def __init__(self, model, N: int, T: int, Be_max: int, device, sm_count: int, fused_step="auto") -> None:
        rnn = model.rnn.rnn
        self.model = model
        self.lstm = isinstance(rnn, nn.LSTM)
        self.H = H = rnn.hidden_size
        self.G = 4 if self.lstm else 3
        self.S = 5 if self.lstm else 4
        self.GH = self.G * H
        # training steps as one launch: the hidden GEMM with the cell in its epilogue (H a multiple of 64); "auto" takes
        # it for GRUs, where it measured faster than the two launches (LSTM: slower, its epilogue moves 25 % more bytes)
        want = fused_step is True or (fused_step == "auto" and not self.lstm)
        self.fused_step = want and H % 64 == 0
        self.D = model.obs_dim
        self.Dp = pad8(self.D)
        self.T, self.N, self.Be_max = T, N, Be_max
        self.w_ih, self.w_hh = rnn.weight_ih_l0, rnn.weight_hh_l0
        self.b_ih, self.b_hh = rnn.bias_ih_l0, rnn.bias_hh_l0
        bf = dict(dtype=torch.bfloat16, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        GH, R = self.GH, Be_max * T
        self.w_ih_bf = torch.zeros(GH, self.Dp, **bf)
        self.w_hh_bf = torch.zeros(GH, pad8(H), **bf)
        self.head = MLPPlan(model.mlp, H, N, R, device, sm_count)
        # rollout: persistent state and per-step scratch; inputs stored env-major [N, T, Dp] (bf16, normalised)
        self.h = torch.zeros(N, H, **f32)
        self.h_bf = torch.zeros(N, H, **bf)
        self.c = torch.zeros(N, H, **f32) if self.lstm else None
        self.h0 = torch.zeros(N, H, **f32)
        self.c0 = torch.zeros(N, H, **f32) if self.lstm else None
        self.gi_roll = torch.zeros(N, GH, **f32)
        self.gh_roll = torch.zeros(N, GH, **f32)
        self.x = torch.zeros(N * T, self.Dp, **bf)
        self.x_last = torch.zeros(N, self.Dp, **bf)
        self.h_scratch = torch.zeros(N, H, **f32)
        self.hbf_scratch = torch.zeros(N, H, **bf)
        self.c_scratch = torch.zeros(N, H, **f32) if self.lstm else None
        # minibatch (env-major rows e * T + t)
        self.gi = torch.zeros(R, GH, **f32)
        self.gh_step = torch.zeros(Be_max, GH, **f32)
        self.hprev = torch.zeros(R, H, **f32)
        self.hprev_bf = torch.zeros(R, H, **bf)
        self.cprev = torch.zeros(R, H, **f32) if self.lstm else None
        self.c_step = torch.zeros(Be_max, H, **f32) if self.lstm else None
        self.hout_bf = torch.zeros(R, H, **bf)
        self.save = torch.zeros(R, self.S * H, **f32)
        self.dh_head = torch.zeros(R, H, **f32)
        self.dgi = torch.zeros(R, GH, **bf)
        self.dgh = None if self.lstm else torch.zeros(R, GH, **bf)
        self.dh_direct = [torch.zeros(Be_max, H, **f32) for _ in range(2)] if not self.lstm else [None, None]
        self.dh_gemm = [torch.zeros(Be_max, H, **f32) for _ in range(2)]
        self.dc = [torch.zeros(Be_max, H, **f32) for _ in range(2)] if self.lstm else [None, None]
        self.bwd_blocks = ext().rnn_bwd_blocks(Be_max)
        # bias-gradient column sums: one row per backward-cell block, accumulated over the T steps of a sweep
        self.cs_gi = torch.zeros(self.bwd_blocks, GH, **f32)
        self.cs_gh = None if self.lstm else torch.zeros(self.bwd_blocks, GH, **f32)
        self.splits_ih = wgrad_splits(GH, self.D, R, sm_count)
        self.splits_hh = wgrad_splits(GH, H, R, sm_count)
        self.part_ih = torch.zeros(self.splits_ih, GH, self.D, **f32)
        self.part_hh = torch.zeros(self.splits_hh, GH, H, **f32)

    def refresh_shadows(self) -> None:
        C = ext()
        C.to_bf16_padded(self.w_ih.data, self.w_ih_bf, self.w_ih_bf.shape[1])
        C.to_bf16_padded(self.w_hh.data, self.w_hh_bf, self.w_hh_bf.shape[1])
        self.head.refresh_shadows()

    def reduce_segments(self, head_bias_partial, head_parts: int) -> dict[int, tuple]:
        segs = self.head.reduce_segments(head_bias_partial, head_parts)
        parts = self.bwd_blocks
        segs[id(self.w_ih)] = (self.part_ih, self.splits_ih, self.w_ih.numel())
        segs[id(self.w_hh)] = (self.part_hh, self.splits_hh, self.w_hh.numel())
        segs[id(self.b_ih)] = (self.cs_gi, parts, self.b_ih.numel())
        segs[id(self.b_hh)] = (self.cs_gi if self.lstm else self.cs_gh, parts, self.b_hh.numel())
        return segs

    def shadows(self) -> dict[int, torch.Tensor]:
        out = {id(lin.weight): wb for lin, wb in zip(self.head.linears, self.head.w_bf16)}
        out[id(self.w_ih)] = self.w_ih_bf
        out[id(self.w_hh)] = self.w_hh_bf
        return out

    # ---- rollout step ----------------------------------------------------------------------------------------------
    def step(self, x_t: torch.Tensor, ld_x: int, status, h_out=None, hbf_out=None, c_out=None) -> None:
        """One cell step on the persistent state from the normalised input rows ``x_t`` (pitch ``ld_x``). Writes the
        new state in place unless outputs are given (the state is then left unchanged)."""
        C = ext()
        N, H, GH = self.N, self.H, self.GH
        G.gemm(x_t, ld_x, False, self.w_ih_bf, self.Dp, False, N, GH, self.D, G.EPI_F32, self.gi_roll, GH,
               bias=self.b_ih.data, status=status)
        G.gemm(self.h_bf, H, False, self.w_hh_bf, self.w_hh_bf.shape[1], False, N, GH, H, G.EPI_F32, self.gh_roll, GH,
               bias=self.b_hh.data, status=status)
        h_out = self.h if h_out is None else h_out
        hbf_out = self.h_bf if hbf_out is None else hbf_out
        c_out = self.c if c_out is None else c_out
        C.rnn_cell_fwd(N, H, self.lstm, self.gi_roll, GH, self.gh_roll, GH, self.h, H, self.c, H, h_out, H, hbf_out, H,
                       c_out, H, None, None, 0, None, 0, None, 0, None, 0)

    # ---- sequences --------------------------------------------------------------------------------------------------
    # A sequence is L steps of Be environments. Its rows are env-major (row e * L + t: PPO minibatches, contiguous env
    # ranges of the rollout) or time-major (row t * Be + e: distillation windows, contiguous step ranges). ``at``
    # gives the first element of step t's rows in a buffer of row width W, and the row pitch of that step.
    @staticmethod
    def _layout(Be: int, L: int, time_major: bool):
        if time_major:
            return lambda buf, t, W: (_view_from(buf, t * Be * W), W)
        return lambda buf, t, W: (_view_from(buf, t * W), L * W)

    def forward_sequence(self, lo: int, Be: int, dones_tm: torch.Tensor, head_out: torch.Tensor, head_ld: int,
                         status, *, L: int | None = None, t0: int = 0, time_major: bool = False, x=None, init=None,
                         carry=None) -> None:
        """Forward of environments ``lo .. lo + Be - 1`` over steps ``t0 .. t0 + L - 1`` (dones read at those absolute
        steps of ``dones_tm`` [T_rollout, N]). ``x``: the sequence's normalised input rows (default: the env-major
        rollout inputs); ``init``: (h, c) state before the first step (default: the state stored at the rollout's
        first step); ``carry``: (h, h_bf16, c) receiving the state after the last step, masked by its dones."""
        C = ext()
        N, H, GH, S = self.N, self.H, self.GH, self.S
        L = self.T if L is None else L
        R = Be * L
        at = self._layout(Be, L, time_major)
        if x is None:
            x = self.x[lo * L : (lo + Be) * L]
        G.gemm(x, self.Dp, False, self.w_ih_bf, self.Dp, False, R, GH, self.D, G.EPI_F32, self.gi, GH,
               bias=self.b_ih.data, status=status)
        if init is None:  # the state stored at the rollout's first step
            init = (self.h0[lo : lo + Be], self.c0[lo : lo + Be] if self.lstm else None)
        C.rnn_mask(Be, H, init[0], H, init[1] if self.lstm else None, H, None, *at(self.hprev, 0, H),
                   *at(self.hprev_bf, 0, H), *(at(self.cprev, 0, H) if self.lstm else (None, 0)))
        for t in range(L):
            nxt = t + 1 < L
            ta = (t0 + t) * N + lo
            if nxt:
                done_t = dones_tm[ta : ta + Be]
                h_next, hbf_next = at(self.hprev, t + 1, H), at(self.hprev_bf, t + 1, H)
                c_next = at(self.cprev, t + 1, H) if self.lstm else (None, 0)
            elif carry is not None:
                done_t = dones_tm[ta : ta + Be]
                h_next, hbf_next = (carry[0], H), (carry[1], H)
                c_next = (carry[2], H) if self.lstm else (None, 0)
            else:
                done_t, h_next, hbf_next, c_next = None, (None, 0), (None, 0), (None, 0)
            c_in = at(self.cprev, t, H) if self.lstm else (None, 0)
            if self.fused_step:
                C.rnn_step_fused(Be, H, self.lstm, *at(self.hprev_bf, t, H), self.w_hh_bf, self.w_hh_bf.shape[1],
                                 self.b_hh.data, *at(self.gi, t, GH), *at(self.hprev, t, H), *c_in, None, 0,
                                 *at(self.hout_bf, t, H), None, 0, done_t, *h_next, *hbf_next, *c_next,
                                 *at(self.save, t, S * H), status)
                continue
            G.gemm(*at(self.hprev_bf, t, H), False, self.w_hh_bf, self.w_hh_bf.shape[1], False, Be, GH, H,
                   G.EPI_F32, self.gh_step, GH, bias=self.b_hh.data, status=status)
            C.rnn_cell_fwd(Be, H, self.lstm, *at(self.gi, t, GH), self.gh_step, GH, *at(self.hprev, t, H), *c_in,
                           None, 0, *at(self.hout_bf, t, H), self.c_step, H, done_t, *h_next, *hbf_next, *c_next,
                           *at(self.save, t, S * H))
        self.head.forward(self.hout_bf, self.head.h_train, R, head_out, head_ld, status)

    def backward_sequence(self, lo: int, Be: int, dones_tm: torch.Tensor, status, *, L: int | None = None,
                          t0: int = 0, time_major: bool = False, x=None) -> None:
        """Backpropagation through the sequence of the last ``forward_sequence`` (same arguments): the head's
        output gradient must be in ``head.d_head``; no gradient enters from after the last step or leaves through
        the initial state. Leaves split-K weight-gradient partials and bias column sums for the segment reduction."""
        C = ext()
        N, H, GH, S = self.N, self.H, self.GH, self.S
        L = self.T if L is None else L
        R = Be * L
        at = self._layout(Be, L, time_major)
        nb = self.bwd_blocks
        if C.rnn_bwd_blocks(Be) < nb:  # a shorter env range writes fewer column-sum rows
            used = C.rnn_bwd_blocks(Be)
            for cs in (self.cs_gi, self.cs_gh):
                if cs is not None:
                    cs[used:].zero_()
        self.head.backward(R, status, x=self.hout_bf, dx_out=self.dh_head)
        dgh = self.dgi if self.lstm else self.dgh
        for t in range(L - 1, -1, -1):
            cur, prev = t & 1, (t + 1) & 1
            last = t == L - 1
            ta = (t0 + t) * N + lo
            C.rnn_cell_bwd(Be, H, self.lstm, *at(self.save, t, S * H),
                           *(at(self.hprev, t, H) if not self.lstm else (None, 0)),
                           *(at(self.cprev, t, H) if self.lstm else (None, 0)),
                           *at(self.dh_head, t, H),
                           None if (last or self.lstm) else self.dh_direct[prev],
                           None if last else self.dh_gemm[prev], H,
                           None if (last or not self.lstm) else self.dc[prev], H,
                           None if last else dones_tm[ta : ta + Be],
                           *at(self.dgi, t, GH),
                           *(at(self.dgh, t, GH) if not self.lstm else (None, 0)),
                           self.dh_direct[cur], H, self.dc[cur], H, self.cs_gi, self.cs_gh, not last)
            if t > 0:  # gradient of the step's input state through W_hh (W_hh [GH, H] read MN-major)
                G.gemm(*at(dgh, t, GH), False, self.w_hh_bf, self.w_hh_bf.shape[1], True, Be, H, GH,
                       G.EPI_F32, self.dh_gemm[cur], H, status=status)
        # weight gradients over all L x Be rows: dW_ih = dgi^T x, dW_hh = dgh^T h_in (split-K partials)
        if x is None:
            x = self.x[lo * L : (lo + Be) * L]
        for part, splits_max, a, b, ldb, ncols in ((self.part_ih, self.splits_ih, self.dgi, x, self.Dp, self.D),
                                                   (self.part_hh, self.splits_hh, dgh, self.hprev_bf, H, H)):
            splits = min(splits_max, (R + 63) // 64)
            if splits < splits_max:
                part[splits:].zero_()
            G.gemm(a, GH, True, b, ldb, True, GH, ncols, R, G.EPI_PARTIAL_F32, part, ncols, splits=splits,
                   split_stride=GH * ncols, status=status)


class RecurrentPPOEngine(EngineBase):
    # ---- capability checks ------------------------------------------------------------------------------------------
    @staticmethod
    def supports_models(actor, critic, alg_cfg: dict) -> str | None:
        for name, m in (("actor", actor), ("critic", critic)):
            reason = rnn_model_reason(name, m)
            if reason:
                return reason
        dist = actor.distribution
        if not isinstance(dist, (GaussianDistribution, HeteroscedasticGaussianDistribution)):
            return "actor distribution is not Gaussian"
        if dist.output_dim > 32:
            return "more than 32 actions"
        if critic.distribution is not None or critic.mlp.linears[-1].out_features != 1:
            return "critic output is not a scalar value"
        rnd_cfg = alg_cfg.get("rnd_cfg")
        if isinstance(rnd_cfg, dict) and str(rnd_cfg.get("activation", "elu")).lower() != "elu":
            return "RND activation is not fused (ELU only)"
        if str(alg_cfg.get("optimizer", "adam")).lower() != "adam":
            return "only Adam is fused"
        return None

    @staticmethod
    def unsupported_reason(alg) -> str | None:
        cfg = {"normalize_advantage_per_mini_batch": alg.normalize_advantage_per_mini_batch,
               "optimizer": getattr(alg, "optimizer_name", "adam")}
        reason = RecurrentPPOEngine.supports_models(alg.actor, alg.critic, cfg)
        if reason is None and alg.rnd is not None:
            reason = rnd_reason(alg.rnd)
        return reason

    # ---- construction -------------------------------------------------------------------------------------------------
    def __init__(self, alg, num_steps_per_env: int, num_envs: int, obs_template=None) -> None:
        self.alg = alg
        self.device = torch.device(alg.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        f32 = dict(dtype=torch.float32, device=dev)
        C = ext()
        self.T, self.N = num_steps_per_env, num_envs
        self.total = self.T * self.N
        self.M, self.E = alg.num_mini_batches, alg.num_learning_epochs
        if not 1 <= self.M <= self.N:
            raise ValueError("num_mini_batches must be between 1 and the number of environments.")
        self.Be_max = max((i + 1) * self.N // self.M - i * self.N // self.M for i in range(self.M))
        self.sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
        self.actor, self.critic = alg.actor, alg.critic
        dist = self.actor.distribution
        self.hetero = isinstance(dist, HeteroscedasticGaussianDistribution)
        self.log_std = dist.std_type == "log"
        self.A = dist.output_dim
        self.std_range, self.log_std_range = dist.std_range, dist.log_std_range
        self.groups_a, self.groups_c = list(self.actor.obs_groups), list(self.critic.obs_groups)
        self.Da, self.Dc = self.actor.obs_dim, self.critic.obs_dim

        # ---- flat parameter arena ----
        self.params = list(dict.fromkeys(chain(self.actor.parameters(), self.critic.parameters())))
        actor_ids = {id(p) for p in self.actor.parameters()}
        self.param_group = [0 if id(p) in actor_ids else 1 for p in self.params]
        if self.param_group != sorted(self.param_group):
            raise RuntimeError("fused engine: actor parameters must precede critic parameters")
        self.rnd = alg.rnd
        if self.rnd is not None:  # the predictor: a third parameter group (own learning rate, no clipping)
            rnd_params = list(self.rnd.predictor.parameters())
            self.params += rnd_params
            self.param_group += [_GROUP_RND] * len(rnd_params)
        self.offsets, off = [], 0
        for p in self.params:
            self.offsets.append(off)
            off += p.numel()
        self.n_params = off
        self.flat = torch.zeros(self.n_params, **f32)
        for p, o in zip(self.params, self.offsets):
            self.flat[o : o + p.numel()].copy_(p.data.reshape(-1))
            p.data = self.flat[o : o + p.numel()].view_as(p)
        n_actor = sum(p.numel() for p, g in zip(self.params, self.param_group) if g == 0)
        n_ac = sum(p.numel() for p, g in zip(self.params, self.param_group) if g != _GROUP_RND)
        self.group_ranges = [0, n_actor, n_actor, n_ac]
        if self.rnd is not None:
            self.group_ranges += [n_ac, self.n_params]
        self.n_ex = (self.n_params + _TAIL + 3) // 4 * 4
        self.exp_avg = torch.zeros(self.n_params, **f32)
        self.exp_avg_sq = torch.zeros(self.n_params, **f32)
        self.world, self.rank = alg.gpu_world_size, alg.gpu_global_rank
        self.timeout_ns = int(alg.b200_cfg["comm_timeout_ms"] * 1e6)
        self.comm = None
        self._peer_reduced = None  # set for the two-shot exchange
        self._kl_offset = self.n_params + 3  # index of the KL statistic in the exchanged vector
        if self.world > 1:
            from ..parallel import PeerExchange

            big = max((t.numel() for t in self.rnd.state_dict().values()), default=0) if self.rnd is not None else 0
            dmax = max(self.Da, self.Dc, self.rnd.num_states if self.rnd is not None else 0)
            small = max(4 * self.n_params, 4 * big, 8 * (2 + 2 * dmax), 4096)
            self.comm = PeerExchange.create(self.n_ex, small, rank=self.rank, world=self.world, device=dev,
                                            timeout_ms=alg.b200_cfg["comm_timeout_ms"])
            from ..algorithms.ppo import use_two_shot

            # two-shot exchange: the ranks' reduced buffers; the KL statistic is read from its owner's shard
            if use_two_shot(alg.b200_cfg, self.world):
                self._peer_reduced = self.comm.peer_reduced

            self.send = self.comm.send
        else:
            buf = torch.zeros(self.n_ex, **f32)
            self.send = [buf, buf]
        self.grads = torch.zeros(self.n_ex, **f32)
        # learning-rate slots: 0 = PPO optimizer (adaptive), 2 = RND predictor optimizer; one step counter per group
        lr_rnd = self.rnd.optimizer.param_groups[0]["lr"] if self.rnd is not None else 0.0
        self.lr = torch.tensor([alg._learning_rate, alg._learning_rate, lr_rnd], **f32)
        self.step = torch.zeros(3, dtype=torch.int64, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=dev)
        self.barrier = torch.zeros(4, dtype=torch.int32, device=dev)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=dev)
        self.rng_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self.rng_ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.seed = int(torch.initial_seed() % (2**62))

        # ---- networks ----
        fused = alg.b200_cfg["rnn_fused_step"]
        self.net_a = _RecurrentNet(self.actor, self.N, self.T, self.Be_max, dev, self.sm_count, fused)
        self.net_c = _RecurrentNet(self.critic, self.N, self.T, self.Be_max, dev, self.sm_count, fused)
        self.nets = (self.net_a, self.net_c)
        for net in self.nets:
            net.refresh_shadows()
        self.head_cols = self.net_a.head.head_cols
        # RND: the predictor trains on a minibatch's env-major rows plus one row standing for the zero-padded
        # trajectory entries of upstream's recurrent minibatch (see _minibatch)
        self.rnd_part = None
        self.intrinsic_for_logger = None
        if self.rnd is not None:
            self.rnd_part = RndPart(self, self.rnd, self.N, self.T, self.Be_max * self.T + 1, dev, self.sm_count)
            for plan in self.rnd_part.plans:
                plan.refresh_shadows()
            self.intrinsic_for_logger = self.rnd_part.intrinsic
            alg.intrinsic_rewards = self.rnd_part.intrinsic

        # ---- rollout arena (time-major rows t * N + n, as the GAE kernel expects) ----
        T, N, A = self.T, self.N, self.A
        self.obs_a = torch.zeros(T * N, (self.Da + 3) // 4 * 4, **f32)[:, : self.Da]
        self.obs_c = torch.zeros(T * N, (self.Dc + 3) // 4 * 4, **f32)[:, : self.Dc]
        self.st_actions = torch.zeros(T * N, A, **f32)
        self.st_mean = torch.zeros(T * N, A, **f32)
        self.st_std = torch.zeros(T * N, A, **f32)
        self.st_logp = torch.zeros(T * N, **f32)
        self.st_values = torch.zeros(T * N, **f32)
        self.st_rewards = torch.zeros(T * N, **f32)
        self.st_dones = torch.zeros(T * N, **f32)
        self.st_returns = torch.zeros(T * N, **f32)
        self.st_adv = torch.zeros(T * N, **f32)
        self.actions_out = torch.zeros(N, A, **f32)
        self.last_values = torch.zeros(N, **f32)
        self.gae_partial = torch.zeros(2 * C.gae_blocks(N), dtype=torch.float64, device=dev)
        self.t = 0
        if self.rnd is not None:
            Dr = self.rnd_part.Dr
            # raw RND states, time-major, plus one zero row at T * N: the state of every zero-padded entry
            self.obs_r = torch.zeros(T * N + 1, (Dr + 3) // 4 * 4, **f32)[:, :Dr]
            self.rnd_idx_out = torch.zeros(self.Be_max * T + 1, dtype=torch.int32, device=dev)
            self.rnd_pad = torch.zeros(1, **f32)  # padded entries of the current minibatch (weight of the zero row)

        # ---- minibatch: storage row of every env-major minibatch row (e, t) -> t * N + lo + e ----
        self.mb_idx = []
        for i in range(self.M):
            lo, hi = i * N // self.M, (i + 1) * N // self.M
            e = torch.arange(lo, hi, device=dev, dtype=torch.int64)
            t = torch.arange(T, device=dev, dtype=torch.int64)
            self.mb_idx.append((t[None, :] * N + e[:, None]).reshape(-1).to(torch.int32).contiguous())
        self.mb_idx_r = None
        if self.rnd is not None:
            pad_row = torch.full((1,), T * N, dtype=torch.int32, device=dev)
            self.mb_idx_r = [torch.cat([idx, pad_row]).contiguous() for idx in self.mb_idx]
        R_max = self.Be_max * T
        self.value_train = torch.zeros(R_max, 1, **f32)
        self.d_value = self.net_c.head.d_head
        self.loss_blocks = C.ppo_loss_blocks(R_max)
        self.stats_partial = torch.zeros(self.loss_blocks, _TAIL, **f32)
        self.dhead_colsum = torch.zeros(self.loss_blocks, self.head_cols, **f32)
        self.dvalue_colsum = torch.zeros(self.loss_blocks, 1, **f32)
        self.dstd_partial = torch.zeros(self.loss_blocks, A, **f32)
        self.loss_acc = torch.zeros(_TAIL, **f32)
        self.adv_per_mb = bool(alg.normalize_advantage_per_mini_batch)
        self.adv_mb = torch.zeros(R_max, **f32) if self.adv_per_mb else None
        self.adv_mb_partial = (torch.zeros(2 * C.adv_gather_blocks(R_max), dtype=torch.float64, device=dev)
                               if self.adv_per_mb else None)

        # ---- gradient reduction plan ----
        seg = {}
        seg.update(self.net_a.reduce_segments(self.dhead_colsum, self.loss_blocks))
        seg.update(self.net_c.reduce_segments(self.dvalue_colsum, self.loss_blocks))
        if self.rnd is not None:
            seg.update(self.rnd_part.reduce_segments())
        if not self.hetero:
            std_p = dist.std_param if dist.std_type == "scalar" else dist.log_std_param
            seg[id(std_p)] = (self.dstd_partial, self.loss_blocks, A)
        srcs, parts, ns, offs = [], [], [], []
        for p, o in zip(self.params, self.offsets):
            if id(p) not in seg:
                raise RuntimeError("fused recurrent engine: parameter without a gradient source")
            buf, nparts, n = seg[id(p)]
            srcs.append(buf)
            parts.append(nparts)
            ns.append(n)
            offs.append(o)
        srcs.append(self.stats_partial)
        parts.append(self.loss_blocks)
        ns.append(_TAIL)
        offs.append(self.n_params)
        self.reduce_plan, self.reduce_nseg, self.reduce_chunks = C.make_reduce_plan(srcs, parts, ns, offs)

        # ---- Adam plan ----
        shadows = {}
        for net in self.nets:
            shadows.update(net.shadows())
        if self.rnd is not None:
            pp = self.rnd_part.plan_p
            shadows.update({id(lin.weight): wb for lin, wb in zip(pp.linears, pp.w_bf16)})
        t_off, t_num, t_grp, t_rows, t_cols, t_sh, t_ld = [], [], [], [], [], [], []
        for p, o, g in zip(self.params, self.offsets, self.param_group):
            sh = shadows.get(id(p))
            t_off.append(o)
            t_num.append(p.numel())
            t_grp.append(g)
            t_rows.append(p.shape[0] if sh is not None else 1)
            t_cols.append(p.shape[1] if sh is not None else p.numel())
            t_sh.append(sh)
            t_ld.append(sh.shape[1] if sh is not None else 0)
        t_off.append(self.n_params)
        t_num.append(_TAIL)
        t_grp.append(-1)
        t_rows.append(1)
        t_cols.append(_TAIL)
        t_sh.append(None)
        t_ld.append(0)
        self.adam_tensors, self.adam_chunks, self.adam_nchunks = C.make_adam_plan(t_off, t_num, t_grp, t_rows, t_cols,
                                                                                  t_sh, t_ld, self.flat)
        self.adam_grid = C.adam_grid(dev.index)
        self.norm_partial = torch.zeros(self.adam_grid * 4, **f32)
        group0 = alg.optimizer.param_groups[0]
        b1, b2 = group0.get("betas", (0.9, 0.999))
        self.betas = (float(b1), float(b2))
        self.adam_eps = float(group0.get("eps", 1e-8))
        if float(group0.get("weight_decay", 0.0)) != 0.0 or group0.get("amsgrad", False):
            raise ValueError("fused Adam supports weight_decay=0 and amsgrad=False")
        self.adam_max_norm = [alg.max_grad_norm, alg.max_grad_norm]
        self.adam_beta1, self.adam_beta2 = [self.betas[0]] * 2, [self.betas[1]] * 2
        self.adam_eps_g, self.adam_lr_index = [self.adam_eps] * 2, [0, 0]
        if self.rnd is not None:
            rb1, rb2, reps = self.rnd_part.adam_hparams()
            self.adam_max_norm.append(0.0)
            self.adam_beta1.append(rb1)
            self.adam_beta2.append(rb2)
            self.adam_eps_g.append(reps)
            self.adam_lr_index.append(2)

        self._alloc_norm_scratch("actor", self.total, self.Da)
        self._alloc_norm_scratch("critic", self.total, self.Dc)
        self.use_graphs = bool(alg.b200_cfg["graphs"])
        self._update_graph = None
        self._updates_done = 0
        self._init_base()

    # ---- learning rate / logging ---------------------------------------------------------------------------------------
    def learning_rate(self) -> float:
        return float(HostTransfers.read(self.lr[0:1], "learning_rate")[0])

    def set_learning_rate(self, value: float) -> None:
        self.lr[0].fill_(value)

    def action_std(self) -> torch.Tensor:
        if self.hetero:
            return self.st_std.mean(dim=0)
        return self.actor.distribution.current_std().detach()

    # ---- rollout ------------------------------------------------------------------------------------------------------
    def _std_param(self):
        d = self.actor.distribution
        return None if self.hetero else (d.std_param if d.std_type == "scalar" else d.log_std_param)

    def act(self, obs) -> torch.Tensor:
        if self.t >= self.T:
            raise OverflowError("Rollout buffer overflow! You should call clear() before adding new transitions.")
        C = ext()
        N, T, t = self.N, self.T, self.t
        rows = slice(t * N, (t + 1) * N)
        if self.rnd is not None:
            if t == 0 and not torch.cuda.is_current_stream_capturing():
                self.rnd_part.prepare()
            # store the raw RND state (the bf16 copy in the scratch row buffer is not used)
            rp = self.rnd_part.plan_p
            C.prep_obs(self._group_tensors(obs, self.rnd_part.groups), self.obs_r[rows], self.obs_r.stride(0),
                       rp.x_roll, rp.x_roll.shape[1], None, None, 0.0)
        for net, model, groups, arena in ((self.net_a, self.actor, self.groups_a, self.obs_a),
                                          (self.net_c, self.critic, self.groups_c, self.obs_c)):
            mean, std, eps = self._norm_tensors(model)
            x_t = _view_from(net.x, t * net.Dp)
            C.prep_obs(self._group_tensors(obs, groups), arena[rows], arena.stride(0), x_t, T * net.Dp, mean, std, eps)
            if t == 0:  # the state every trajectory of this rollout that does not start at a done resumes from
                net.h0.copy_(net.h)
                if net.lstm:
                    net.c0.copy_(net.c)
            net.step(x_t, T * net.Dp, self.status)
        pa, pc = self.net_a.head, self.net_c.head
        pa.forward(self.net_a.h_bf, pa.h_roll, N, pa.out_roll, pa.out_roll.shape[1], self.status)
        std_param = self._std_param()
        C.gaussian_sample(pa.out_roll, pa.out_roll.shape[1], N, self.A, self.hetero, self.log_std,
                          None if std_param is None else std_param.data, self.std_range[0], self.std_range[1],
                          self.log_std_range[0], self.log_std_range[1], self.seed, self.rng_counter, self.rng_ticket,
                          self.st_actions[rows], self.st_mean[rows], self.st_std[rows], self.st_logp[rows],
                          self.actions_out)
        pc.forward(self.net_c.h_bf, pc.h_roll, N, self.st_values[rows].view(N, 1), 1, self.status)
        return self.actions_out

    def process_env_step(self, obs, rewards, dones, extras) -> None:
        C = ext()
        N, t = self.N, self.t
        rows = slice(t * N, (t + 1) * N)
        timeouts = extras.get("time_outs") if isinstance(extras, dict) else None
        if timeouts is not None:
            timeouts = timeouts.to(self.device).reshape(-1)
        intrinsic = self.rnd_part.intrinsic_reward(self, obs, t) if self.rnd is not None else None
        C.process_step(rewards.reshape(-1).float(), intrinsic, dones.reshape(-1), timeouts, self.st_values[rows],
                       self.alg.gamma, self.st_rewards[rows], self.st_dones[rows], self.nonfinite)
        done_f = self.st_dones[rows]
        for net in self.nets:  # reset the state of finished episodes
            H = net.H
            C.rnn_mask(N, H, net.h, H, net.c, H, done_f, net.h, H, net.h_bf, H, net.c, H)
        self.t += 1

    def _before_replay(self) -> None:
        if self.rnd is not None:
            self.rnd_part.prepare()

    def compute_returns(self, obs) -> None:
        C = ext()
        net = self.net_c
        mean, std, eps = self._norm_tensors(self.critic)
        C.prep_obs(self._group_tensors(obs, self.groups_c), None, self.Dc, net.x_last, net.Dp, mean, std, eps)
        # value of the last observation from the current state, which stays untouched
        net.step(net.x_last, net.Dp, self.status, h_out=net.h_scratch, hbf_out=net.hbf_scratch, c_out=net.c_scratch)
        net.head.forward(net.hbf_scratch, net.head.h_roll, self.N, self.last_values.view(self.N, 1), 1, self.status)
        C.gae(self.st_rewards, self.st_dones, self.st_values, self.last_values, self.st_returns, self.st_adv, self.T,
              self.N, self.alg.gamma, self.alg.lam, self.gae_partial)
        if self.total > 1 and not self.adv_per_mb:
            C.adv_normalize(self.st_adv, self.gae_partial, C.gae_blocks(self.N))
        self.t = 0

    # ---- update -------------------------------------------------------------------------------------------------------
    def _minibatch(self, i: int) -> None:
        C = ext()
        lo = i * self.N // self.M
        Be = (i + 1) * self.N // self.M - lo
        R = Be * self.T
        used = C.ppo_loss_blocks(R)
        if used < self.loss_blocks:
            for buf in (self.stats_partial, self.dhead_colsum, self.dvalue_colsum, self.dstd_partial):
                buf[used:].zero_()
        pa = self.net_a.head
        self.net_a.forward_sequence(lo, Be, self.st_dones, pa.out_train, pa.out_train.shape[1], self.status)
        self.net_c.forward_sequence(lo, Be, self.st_dones, self.value_train, 1, self.status)
        std_param = self._std_param()
        alg = self.alg
        adv_override = None
        if self.adv_per_mb and R > 1:
            C.adv_gather_stats(self.st_adv, self.mb_idx[i], R, self.adv_mb, self.adv_mb_partial, self.status)
            C.adv_normalize(self.adv_mb[:R], self.adv_mb_partial, C.adv_gather_blocks(R))
            adv_override = self.adv_mb
        C.ppo_loss(R, self.A, self.hetero, self.log_std, pa.out_train, pa.out_train.shape[1], self.value_train, 1,
                   None if std_param is None else std_param.data, self.std_range[0], self.std_range[1],
                   self.log_std_range[0], self.log_std_range[1], self.mb_idx[i], self.st_actions, self.st_mean,
                   self.st_std, self.st_logp, self.st_adv, self.st_returns, self.st_values, adv_override,
                   alg.clip_param,
                   alg.value_loss_coef, alg.entropy_coef, alg.use_clipped_value_loss, pa.d_head, pa.d_head.shape[1],
                   self.d_value, self.d_value.shape[1], self.stats_partial, self.dhead_colsum, self.dvalue_colsum,
                   None if self.hetero else self.dstd_partial, 1, False, None, None, 0.0, self.status)
        self.net_a.backward_sequence(lo, Be, self.st_dones, self.status)
        self.net_c.backward_sequence(lo, Be, self.st_dones, self.status)
        if self.rnd is not None:
            self._rnd_minibatch(i, lo, Be)
        C.reduce_segments(self.reduce_plan, self.reduce_nseg, self.reduce_chunks, self.send[0], self.send[1],
                          self.epoch, False)
        adaptive = alg.desired_kl is not None and alg.schedule == "adaptive"
        kl = self.grads[self.n_params + 3 : self.n_params + 4]
        peers = self.comm.peer_send if self.comm is not None else None
        flags = self.comm.peer_flags if self.comm is not None else None
        C.adam_step(self.flat, self.send[0], self.send[1], self.grads, self.exp_avg, self.exp_avg_sq,
                    self.adam_tensors, self.adam_chunks, self.adam_nchunks, self.adam_max_norm, self.adam_beta1,
                    self.adam_beta2, self.adam_eps_g, self.adam_lr_index, self.lr, None, self.step, adaptive, kl, float(alg.desired_kl or 0.0), 1e-5, 1e-2, self.world, self.rank, peers, flags,
                    self.epoch, self.timeout_ns, self.norm_partial, self.barrier, self.status, None, self.adam_grid,
                    self.group_ranges, self.n_ex, self._peer_reduced, self._kl_offset)
        self.loss_acc.add_(self.grads[self.n_params : self.n_params + _TAIL])

    def _rnd_minibatch(self, i: int, lo: int, Be: int) -> None:
        """Predictor step of minibatch ``i`` as upstream's ``rnd.compute_loss`` on the recurrent minibatch: its
        observations are the padded trajectories ``[T, trajectories]``, so the MSE averages over the real entries
        (the env range's ``Be x T`` rows) and the zero-padded ones, which all share the normalised zero state. Every
        environment has one trajectory plus one per done before its last step, each padded to ``T`` entries: the
        zero row's weight is ``T x`` that done count, computed on the device."""
        C = ext()
        part = self.rnd_part
        rows = Be * self.T + 1
        part.zero_tails(rows)
        mean_r, std_r, eps_r = self._norm_views(self.rnd.state_normalizer)
        rp = part.plan_p
        C.gather_minibatch(rows, 0, self.total + 1, None, 0, self.mb_idx_r[i], self.rnd_idx_out, [self.obs_r],
                           [mean_r], [std_r], eps_r if mean_r is not None else 0.0, [rp.x_train], [rp.x_train.shape[1]],
                           self.status, 1, [rows], [None], [None])
        C.rnn_pad_entries(self.st_dones, self.T, self.N, lo, Be, self.rnd_pad)
        part.train(rows, self.status, self.rnd_pad)

    def _update_body(self) -> None:
        self.loss_acc.zero_()
        if self.rnd is not None:
            self.rnd_part.loss_acc.zero_()
        for _ in range(self.E):
            for i in range(self.M):
                self._minibatch(i)
        self._normalizer_update("actor", self.actor, self.obs_a, self.total, self.Da)
        self._normalizer_update("critic", self.critic, self.obs_c, self.total, self.Dc)
        if self.rnd is not None:
            self.rnd_part.normalizer_update(self, self.obs_r, self.total)

    def update(self) -> dict[str, float]:
        if self.use_graphs and self._updates_done >= 1:
            if self._update_graph is None:
                self._update_graph = self._capture(self._update_body)
            self._update_graph.replay()
        else:
            self._update_body()
        self._updates_done += 1
        n = float(self.E * self.M)
        stats = [v / n for v in HostTransfers.read(self.loss_acc, "loss_stats")]
        self._check_status()
        out = {"value": stats[1], "surrogate": stats[0], "entropy": stats[2]}
        if self.rnd is not None:
            out["rnd"] = float(HostTransfers.read(self.rnd_part.loss_acc, "rnd_loss")[0]) / n
        return out

    # ---- rollout import (tests) -----------------------------------------------------------------------------------------
    def load_rollout(self, storage, h0_actor: torch.Tensor, h0_critic: torch.Tensor, c0_actor=None,
                     c0_critic=None) -> None:
        """Take a filled recurrent :class:`RolloutStorage` ([T, N, ...]) and the rollout's initial states."""
        C = ext()
        T, N = self.T, self.N
        obs = storage.observations.flatten(0, 1)
        for net, model, groups, arena, h0, c0 in ((self.net_a, self.actor, self.groups_a, self.obs_a, h0_actor,
                                                   c0_actor),
                                                  (self.net_c, self.critic, self.groups_c, self.obs_c, h0_critic,
                                                   c0_critic)):
            arena.copy_(torch.cat([obs[g] for g in groups], dim=-1))
            mean, std, eps = self._norm_tensors(model)
            for t in range(T):
                C.prep_obs([arena[t * N : (t + 1) * N]], None, net.D, _view_from(net.x, t * net.Dp), T * net.Dp,
                           mean, std, eps)
            net.h0.copy_(h0)
            if net.lstm:
                net.c0.copy_(c0)
        if self.rnd is not None:
            self.obs_r[: T * N].copy_(torch.cat([obs[g] for g in self.rnd_part.groups], dim=-1))
        mean, std = storage.distribution_params[0], storage.distribution_params[1]
        self.st_actions.copy_(storage.actions.reshape(T * N, -1))
        self.st_mean.copy_(mean.reshape(T * N, -1))
        self.st_std.copy_(std.reshape(T * N, -1).expand(T * N, self.A))
        self.st_logp.copy_(storage.actions_log_prob.reshape(-1))
        self.st_values.copy_(storage.values.reshape(-1))
        self.st_rewards.copy_(storage.rewards.reshape(-1))
        self.st_dones.copy_(storage.dones.reshape(-1).float())
        self.st_returns.copy_(storage.returns.reshape(-1))
        self.st_adv.copy_(storage.advantages.reshape(-1))

    # ---- checkpoints --------------------------------------------------------------------------------------------------
    def _optimizer_of(self, g: int):
        return self.rnd.optimizer if g == _GROUP_RND else self.alg.optimizer

    def sync_to_torch(self) -> None:
        """Expose the device optimizer state through the ``torch.optim.Adam`` objects (parameters are already views)."""
        steps = HostTransfers.read(self.step, "adam_step")
        for p, o, g in zip(self.params, self.offsets, self.param_group):
            if steps[g] == 0:
                continue
            n = p.numel()
            self._optimizer_of(g).state[p] = {"step": torch.tensor(float(steps[g])),
                                              "exp_avg": self.exp_avg[o : o + n].view_as(p),
                                              "exp_avg_sq": self.exp_avg_sq[o : o + n].view_as(p)}
        lrs = HostTransfers.read(self.lr, "learning_rate")
        for group in self.alg.optimizer.param_groups:
            group["lr"] = lrs[0]
        self.alg._learning_rate = lrs[0]
        if self.rnd is not None:
            for group in self.rnd.optimizer.param_groups:
                group["lr"] = lrs[2]

    def sync_from_torch(self) -> None:
        """Pull loaded weights / optimizer state into the device arena and refresh the bf16 shadows."""
        for p, o, g in zip(self.params, self.offsets, self.param_group):
            n = p.numel()
            if p.data.data_ptr() != self.flat[o : o + n].data_ptr():
                self.flat[o : o + n].copy_(p.data.reshape(-1))
                p.data = self.flat[o : o + n].view_as(p)
            opt = self._optimizer_of(g)
            st = opt.state.get(p)
            if st:
                self.exp_avg[o : o + n].copy_(st["exp_avg"].reshape(-1))
                self.exp_avg_sq[o : o + n].copy_(st["exp_avg_sq"].reshape(-1))
                self.step[g] = int(float(st["step"]))
                opt.state[p] = {"step": st["step"], "exp_avg": self.exp_avg[o : o + n].view_as(p),
                                "exp_avg_sq": self.exp_avg_sq[o : o + n].view_as(p)}
        self.lr[0:2].fill_(float(self.alg.optimizer.param_groups[0]["lr"]))
        if self.rnd is not None:
            self.lr[2] = self.rnd_part.learning_rate()
        self._refresh_shadows()

    def _refresh_shadows(self) -> None:
        for net in self.nets:
            net.refresh_shadows()
        if self.rnd is not None:
            for plan in self.rnd_part.plans:
                plan.refresh_shadows()

    def broadcast_parameters(self) -> None:
        """Make every rank start from rank 0's parameters and normaliser buffers."""
        extra = [] if self.rnd is None else self.rnd_part.broadcast_modules()
        if self.comm is not None:
            self.comm.broadcast_(self.flat, status=self.status)
            for model in [self.actor, self.critic] + ([self.rnd.predictor] if self.rnd is not None else []):
                for b in model.buffers():
                    self.comm.broadcast_(b, status=self.status)
            for m in extra:
                for t in m.state_dict().values():
                    self.comm.broadcast_(t, status=self.status)
            self._check_status()
        else:
            for model in [self.actor, self.critic] + ([self.rnd] if self.rnd is not None else []):
                for t in model.state_dict().values():
                    torch.distributed.broadcast(t, src=0)
        self._refresh_shadows()


__all__ = ["RecurrentPPOEngine", "rnn_model_reason"]
