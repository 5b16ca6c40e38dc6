"""Fused CUDA engines of :class:`tt_rsl_rl_b200.algorithms.Distillation` (behaviour cloning of a teacher).

Device-resident state: the student's trainable parameters in a flat fp32 arena (the ``nn.Parameter``s are views, so
checkpoints are unchanged), flat Adam moments, bf16 weight shadows of student and teacher, and a rollout arena holding
per step the raw student observations (for the normaliser update), the student's *normalised bf16 GEMM input* and the
teacher's actions. The teacher is an MLP or a recurrent model (GRU / LSTM with its own rollout state, reset at dones);
it only runs inference.

:class:`DistillationEngine` (MLP student). Per iteration:

* ``act``: observation concat + normalisation of both models, student forward with Philox Gaussian sampling (the
  environment action), teacher forward into the target arena; ``process_env_step`` only checks rewards for NaN/Inf.
* ``update``: for each epoch and each of the ``T`` stored steps, in storage order (``distillation.py:149-179``):
  student forward straight from the stored bf16 input, the loss-gradient kernel (MSE or Huber, output-bias column
  sums, loss sum), backward GEMMs, and a segment reduction that *adds* the step's gradient to the window's sum; every
  ``gradient_length`` steps the fused (exchange +) clip + Adam kernel applies the window. Steps left over at the end
  are accumulated but never applied, as upstream. Then the student normaliser update. From the second call on the
  whole update is one CUDA graph replay.

:class:`RecurrentDistillationEngine` (GRU / LSTM student) follows the same window rule with the student's state
carried through the rollout steps (truncated backpropagation through time, ``distillation.py:143-201``): every epoch
replays the stored steps from the state the previous update ended with (zero at first); a window's steps run as one
time-major sequence (one input GEMM over all its rows, per step the hidden GEMM and the fused cell, the head over all
rows), its loss gradient flows back through the window's steps only, and the state is reset at dones. A window that
spans two epochs is two sequences whose gradients add up. After the update the rollout continues from the state the
last epoch ended with, as upstream's student keeps its training state.

The student's distribution parameter (``std``) gets no gradient from the deterministic output and, as in
``torch.optim.Adam`` with ``grad=None``, is not updated. The normaliser of the student is not updated during the
rollout, so the stored normalised inputs equal what the update's forward would compute (``distillation.py:190``).
"""

from __future__ import annotations

from itertools import chain

import torch

from ..modules import GaussianDistribution, HeteroscedasticGaussianDistribution
from ..ops import ext
from ..utils.timer import HostTransfers
from .base import EngineBase, elu_mlp_reason
from .mlp_plan import MLPPlan, pad8
from .recurrent_engine import _RecurrentNet, rnn_model_reason


def _mlp_model_reason(name: str, m) -> str | None:
    from ..models import MLPModel

    if type(m) is not MLPModel:
        return f"{name} type {type(m).__name__} is not fused"
    reason = elu_mlp_reason(m)
    if reason:
        return f"{name}: {reason}"
    if m.obs_dim > 1024:
        return f"{name} observation width {m.obs_dim} too large"
    return None


def _teacher_reason(m) -> str | None:
    from ..models import RNNModel

    return rnn_model_reason("teacher", m) if isinstance(m, RNNModel) else _mlp_model_reason("teacher", m)


def window_segments(epochs: int, steps: int, gradient_length: int) -> list[tuple[int, int, int, bool, bool, bool]]:
    """The sequences a recurrent student trains on: ``(epoch, t0, L, first_in_window, train, apply)`` per run of
    ``L`` consecutive steps from ``t0`` that lies in one epoch and one window of ``gradient_length`` steps (windows
    count steps across epochs, as upstream's loss sum does). ``train``: the run belongs to a window that reaches an
    optimizer step (steps left over after the last full window only contribute their loss); ``apply``: the window
    ends with this run."""
    applied = (epochs * steps) // gradient_length * gradient_length
    out, count = [], 0
    for e in range(epochs):
        t = 0
        while t < steps:
            L = min(steps - t, gradient_length - count % gradient_length)
            train = count + L <= applied
            out.append((e, t, L, count % gradient_length == 0, train, train and (count + L) % gradient_length == 0))
            count += L
            t += L
    return out


def _common_reason(alg) -> str | None:
    sd = alg.student.distribution
    if sd is not None and not isinstance(sd, (GaussianDistribution, HeteroscedasticGaussianDistribution)):
        return "student distribution is not Gaussian"
    td = alg.teacher.distribution
    if td is not None and not isinstance(td, (GaussianDistribution, HeteroscedasticGaussianDistribution)):
        return "teacher distribution is not Gaussian"
    A = alg.student.mlp.linears[-1].out_features if sd is None else sd.output_dim
    if A > 32:
        return "more than 32 actions"
    if alg.loss_type not in ("mse", "huber"):
        return f"loss {alg.loss_type} is not fused"
    if str(getattr(alg, "optimizer_name", "adam")).lower() != "adam":
        return "only Adam is fused"
    return None


class DistillationEngine(EngineBase):
    @staticmethod
    def unsupported_reason(alg) -> str | None:
        return (_mlp_model_reason("student", alg.student) or _teacher_reason(alg.teacher) or _common_reason(alg))

    def __init__(self, alg) -> None:
        self._init_common(alg, list(dict.fromkeys(alg.student.mlp.parameters())))
        # the student trains on N rows (one stored step)
        self.plan_s = MLPPlan(self.student.mlp, self.Ds, self.N, self.N, self.device, self.sm_count)
        self.plan_s.refresh_shadows()
        self.head_s = self.plan_s.head_cols
        self._init_teacher()
        self._init_arena(self.N)
        seg = self.plan_s.reduce_segments(self.dhead_colsum, self.mse_blocks)
        shadows = {id(lin.weight): wb for lin, wb in zip(self.plan_s.linears, self.plan_s.w_bf16)}
        self._init_reduce_and_adam(seg, shadows)

    # ---- construction pieces ----------------------------------------------------------------------------------------
    def _init_common(self, alg, params: list) -> None:
        """Sizes, the flat parameter arena of ``params`` (installed as views), the peer exchange and the scalars of
        the fused optimizer."""
        self.alg = alg
        self.device = torch.device(alg.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        storage = alg.storage
        self.T = storage.num_transitions_per_env
        self.N = storage.num_envs
        self.total = self.T * self.N
        self.E = alg.num_learning_epochs
        self.GL = alg.gradient_length
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.student = alg.student
        self.teacher = alg.teacher
        dev = self.device
        f32 = dict(dtype=torch.float32, device=dev)

        sd = self.student.distribution
        self.s_dist = sd
        self.hetero = isinstance(sd, HeteroscedasticGaussianDistribution)
        self.A = self.student.mlp.linears[-1].out_features if sd is None else sd.output_dim
        self.groups_s = list(self.student.obs_groups)
        self.groups_t = list(self.teacher.obs_groups)
        self.Ds = self.student.obs_dim
        self.Dt = self.teacher.obs_dim

        # flat parameter arena (distribution parameters stay outside: no gradient)
        self.params = params
        self.offsets, off = [], 0
        for p in self.params:
            self.offsets.append(off)
            off += p.numel()
        self.n_params = off
        self.flat = torch.zeros(self.n_params, **f32)
        for p, o in zip(self.params, self.offsets):
            self.flat[o : o + p.numel()].copy_(p.data.reshape(-1))
            p.data = self.flat[o : o + p.numel()].view_as(p)
        self.n_ex = (self.n_params + 3) // 4 * 4
        self.exp_avg = torch.zeros(self.n_params, **f32)
        self.exp_avg_sq = torch.zeros(self.n_params, **f32)
        self.world = alg.gpu_world_size
        self.rank = alg.gpu_global_rank
        self.timeout_ns = int(alg.b200_cfg["comm_timeout_ms"] * 1e6)
        self.comm = None
        self._peer_reduced = None  # set for the two-shot exchange
        self._kl_offset = -1  # index of the KL statistic in the exchanged vector (none here)
        if self.world > 1:
            from ..algorithms.ppo import use_two_shot
            from ..parallel import PeerExchange

            t_max = max((t.numel() for t in self.teacher.state_dict().values()), default=0)
            small = max(4 * self.n_params, 4 * t_max, 8 * (2 + 2 * self.Ds), 4096)
            self.comm = PeerExchange.create(self.n_ex, small, rank=self.rank, world=self.world, device=dev,
                                            timeout_ms=alg.b200_cfg["comm_timeout_ms"])
            # two-shot exchange: the ranks' reduced buffers
            if use_two_shot(alg.b200_cfg, self.world):
                self._peer_reduced = self.comm.peer_reduced
            self.send = self.comm.send
        else:
            buf = torch.zeros(self.n_ex, **f32)
            self.send = [buf, buf]
        self.grads = torch.zeros(self.n_ex, **f32)
        self.lr = torch.tensor([alg.learning_rate], **f32)
        self.step = torch.zeros(1, dtype=torch.int64, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=dev)
        self.barrier = torch.zeros(4, dtype=torch.int32, device=dev)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=dev)
        self.rng_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self.rng_ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.seed = int(torch.initial_seed() % (2**62))

    def _init_teacher(self) -> None:
        """The teacher's inference plan: an MLP, or a recurrent net stepping its own rollout state."""
        from ..models import RNNModel

        if isinstance(self.teacher, RNNModel):
            self.tnet = _RecurrentNet(self.teacher, self.N, 1, 1, self.device, self.sm_count)
            self.tnet.refresh_shadows()
            self.plan_t = self.tnet.head
        else:
            self.tnet = None
            self.plan_t = MLPPlan(self.teacher.mlp, self.Dt, self.N, 0, self.device, self.sm_count, train=False)
            self.plan_t.refresh_shadows()
        self.head_t = self.plan_t.head_cols

    def _init_arena(self, train_rows: int) -> None:
        """Rollout arena and the loss-gradient buffers for ``train_rows`` rows per training launch."""
        T, N, A, dev = self.T, self.N, self.A, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        self.obs_s = torch.zeros(T * N, self.Ds, **f32)
        self.x_s = torch.zeros(T * N, pad8(self.Ds), dtype=torch.bfloat16, device=dev)
        self.targets = torch.zeros(T * N, self.head_t, **f32)
        self.st_dones = torch.zeros(T * N, **f32)
        self.actions_out = torch.zeros(N, A, **f32)
        self.scratch_actions = torch.zeros(N, A, **f32)
        self.scratch_mean = torch.zeros(N, A, **f32)
        self.scratch_std = torch.zeros(N, A, **f32)
        self.scratch_logp = torch.zeros(N, **f32)
        self.zero_values = torch.zeros(N, **f32)
        self.scratch_r = torch.zeros(N, **f32)
        self.t = 0
        self.mse_blocks = ext().mse_blocks(train_rows)
        self.loss_partial = torch.zeros(self.mse_blocks, **f32)
        self.dhead_colsum = torch.zeros(self.mse_blocks, self.head_s, **f32)
        self.loss_acc = torch.zeros(1, **f32)
        self.loss_ticket = torch.zeros(1, dtype=torch.int32, device=dev)

    def _init_reduce_and_adam(self, seg: dict, shadows: dict) -> None:
        """Segment-reduction plan of the student's gradient sources and the Adam plan (one group, optional clip)."""
        C = ext()
        srcs, parts, ns, offs = [], [], [], []
        for p, o in zip(self.params, self.offsets):
            if id(p) not in seg:
                raise RuntimeError("fused distillation engine: parameter without a gradient source")
            buf, nparts, n = seg[id(p)]
            srcs.append(buf)
            parts.append(nparts)
            ns.append(n)
            offs.append(o)
        self.reduce_plan, self.reduce_nseg, self.reduce_chunks = C.make_reduce_plan(srcs, parts, ns, offs)
        t_rows, t_cols, t_sh, t_ld = [], [], [], []
        for p in self.params:
            sh = shadows.get(id(p))
            t_rows.append(p.shape[0] if sh is not None else 1)
            t_cols.append(p.shape[1] if sh is not None else p.numel())
            t_sh.append(sh)
            t_ld.append(sh.shape[1] if sh is not None else 0)
        self.adam_tensors, self.adam_chunks, self.adam_nchunks = C.make_adam_plan(
            self.offsets, [p.numel() for p in self.params], [0] * len(self.params), t_rows, t_cols, t_sh, t_ld,
            self.flat)
        self.adam_grid = C.adam_grid(self.device.index)
        self.norm_partial = torch.zeros(self.adam_grid * 4, dtype=torch.float32, device=self.device)
        group0 = self.alg.optimizer.param_groups[0]
        b1, b2 = group0.get("betas", (0.9, 0.999))
        self.betas = (float(b1), float(b2))
        self.adam_eps = float(group0.get("eps", 1e-8))
        if float(group0.get("weight_decay", 0.0)) != 0.0 or group0.get("amsgrad", False):
            raise ValueError("fused Adam supports weight_decay=0 and amsgrad=False")
        self._alloc_norm_scratch("student", self.total, self.Ds)
        self.use_graphs = bool(self.alg.b200_cfg["graphs"])
        self._update_graph = None
        self._updates_done = 0
        self._init_base()

    def _refresh_shadows(self) -> None:
        self.plan_s.refresh_shadows()
        if self.tnet is not None:
            self.tnet.refresh_shadows()
        else:
            self.plan_t.refresh_shadows()

    # ---- learning rate / logging ---------------------------------------------------------------------------------------
    def learning_rate(self) -> float:
        return float(HostTransfers.read(self.lr[0:1], "learning_rate")[0])

    def action_std(self) -> torch.Tensor:
        if self.s_dist is None:
            return torch.zeros(1)
        if self.hetero:
            return self.scratch_std.mean(dim=0)
        return self.s_dist.current_std().detach()

    # ---- rollout ------------------------------------------------------------------------------------------------------
    def _student_forward(self, x_rows: torch.Tensor) -> torch.Tensor:
        """Student output rows of the current step from its normalised input; returns the head output buffer."""
        ps = self.plan_s
        ps.forward(x_rows, ps.h_roll, self.N, ps.out_roll, ps.out_roll.shape[1], self.status)
        return ps.out_roll

    def _teacher_forward(self, obs, out: torch.Tensor) -> None:
        mean_t, std_t, eps_t = self._norm_tensors(self.teacher)
        C = ext()
        if self.tnet is not None:
            net = self.tnet
            C.prep_obs(self._group_tensors(obs, self.groups_t), None, self.Dt, net.x, net.Dp, mean_t, std_t, eps_t)
            net.step(net.x, net.Dp, self.status)
            net.head.forward(net.h_bf, net.head.h_roll, self.N, out, self.head_t, self.status)
            return
        pt = self.plan_t
        C.prep_obs(self._group_tensors(obs, self.groups_t), None, self.Dt, pt.x_roll, pt.x_roll.shape[1], mean_t,
                   std_t, eps_t)
        pt.forward(pt.x_roll, pt.h_roll, self.N, out, self.head_t, self.status)

    def act(self, obs) -> torch.Tensor:
        if self.t >= self.T:
            raise OverflowError("Rollout buffer overflow! You should call clear() before adding new transitions.")
        N, t = self.N, self.t
        rows = slice(t * N, (t + 1) * N)
        C = ext()
        mean_s, std_s, eps_s = self._norm_tensors(self.student)
        x_rows = self.x_s[rows]
        C.prep_obs(self._group_tensors(obs, self.groups_s), self.obs_s[rows], self.Ds, x_rows, x_rows.shape[1], mean_s,
                   std_s, eps_s)
        out = self._student_forward(x_rows)
        self._teacher_forward(obs, self.targets[rows])
        d = self.s_dist
        if d is None:
            return out
        log_std = d.std_type == "log"
        std_param = None if self.hetero else (d.std_param if d.std_type == "scalar" else d.log_std_param)
        C.gaussian_sample(out, out.shape[1], N, self.A, self.hetero, log_std,
                          None if std_param is None else std_param.data, d.std_range[0], d.std_range[1],
                          d.log_std_range[0], d.log_std_range[1], self.seed, self.rng_counter, self.rng_ticket,
                          self.scratch_actions, self.scratch_mean, self.scratch_std, self.scratch_logp,
                          self.actions_out)
        return self.actions_out

    def process_env_step(self, obs, rewards, dones, extras) -> None:
        N, t = self.N, self.t
        done_f = self.st_dones[t * N : (t + 1) * N]
        ext().process_step(rewards.reshape(-1).float(), None, dones.reshape(-1), None, self.zero_values, 0.0,
                           self.scratch_r, done_f, self.nonfinite)
        self._reset_states(done_f)
        self.t += 1

    def _reset_states(self, done_f: torch.Tensor) -> None:
        """Zero the recurrent rollout states of finished episodes (teacher; the student in the recurrent engine)."""
        if self.tnet is not None:
            net = self.tnet
            ext().rnn_mask(self.N, net.H, net.h, net.H, net.c, net.H, done_f, net.h, net.H, net.h_bf, net.H, net.c,
                           net.H)

    def compute_returns(self, obs) -> None:
        """Distillation has no return targets."""

    # ---- update -------------------------------------------------------------------------------------------------------
    def _adam(self) -> None:
        """Apply the window's summed gradient: (exchange +) clip + Adam over the student's parameters."""
        peers = self.comm.peer_send if self.comm is not None else None
        flags = self.comm.peer_flags if self.comm is not None else None
        max_norm = float(self.alg.max_grad_norm or 0.0)
        ext().adam_step(self.flat, self.send[0], self.send[1], self.grads, self.exp_avg, self.exp_avg_sq,
                        self.adam_tensors, self.adam_chunks, self.adam_nchunks, [max_norm], [self.betas[0]],
                        [self.betas[1]], [self.adam_eps], [0], self.lr, None, self.step, False, None, 0.0, 0.0, 0.0,
                        self.world, self.rank, peers, flags, self.epoch, self.timeout_ns, self.norm_partial,
                        self.barrier, self.status, None, self.adam_grid, [0, self.n_params], self.n_ex,
                        self._peer_reduced, self._kl_offset)

    def _reduce(self, accumulate: bool) -> None:
        ext().reduce_segments(self.reduce_plan, self.reduce_nseg, self.reduce_chunks, self.send[0], self.send[1],
                              self.epoch, accumulate)

    def _step(self, t: int, count: int) -> None:
        C = ext()
        N = self.N
        ps = self.plan_s
        x = self.x_s[t * N : (t + 1) * N]
        ps.forward(x, ps.h_train, N, ps.out_train, ps.out_train.shape[1], self.status)
        C.mse_grad(ps.out_train, ps.out_train.shape[1], self.targets[t * N : (t + 1) * N], self.head_t, N, self.A,
                   self.alg.loss_type == "huber", ps.d_head, ps.d_head.shape[1], self.head_s, self.loss_partial,
                   self.dhead_colsum, self.loss_acc, self.loss_ticket, None, 0)
        ps.backward(N, self.status, x=x)
        self._reduce(accumulate=(count - 1) % self.GL != 0)
        if count % self.GL == 0:
            self._adam()

    def _update_body(self) -> None:
        self.loss_acc.zero_()
        count = 0
        for _ in range(self.E):
            for t in range(self.T):
                count += 1
                self._step(t, count)
        self._normalizer_update("student", self.student, self.obs_s, self.total, self.Ds)

    def update(self) -> dict[str, float]:
        if self.use_graphs and self._updates_done >= 1:
            if self._update_graph is None:
                self._update_graph = self._capture(self._update_body)
            self._update_graph.replay()
        else:
            self._update_body()
        self._updates_done += 1
        self.t = 0
        loss = float(HostTransfers.read(self.loss_acc, "loss_stats")[0]) / float(self.E * self.T)
        self._check_status()
        return {"behavior": loss}

    # ---- rollout import (tests / external collectors) -------------------------------------------------------------------
    def load_rollout(self, storage) -> None:
        """Take a filled ``distillation`` :class:`RolloutStorage` (``[T, N, ...]``) as the rollout arena."""
        T, N = self.T, self.N
        obs = storage.observations.flatten(0, 1)
        mean_s, std_s, eps_s = self._norm_tensors(self.student)
        ext().prep_obs([obs[g].contiguous() for g in self.groups_s], self.obs_s, self.Ds, self.x_s,
                       self.x_s.shape[1], mean_s, std_s, eps_s)
        self.targets[:, : self.A].copy_(storage.privileged_actions.reshape(T * N, -1)[:, : self.A])
        self.st_dones.copy_(storage.dones.reshape(-1).float())
        self.t = T

    # ---- checkpoints --------------------------------------------------------------------------------------------------
    def sync_to_torch(self) -> None:
        """Expose the device Adam state through the ``torch.optim`` object (parameters are already views)."""
        opt = self.alg.optimizer
        step = float(HostTransfers.read(self.step[0:1], "adam_step")[0])
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            if step > 0:
                opt.state[p] = {"step": torch.tensor(step), "exp_avg": self.exp_avg[o : o + n].view_as(p),
                                "exp_avg_sq": self.exp_avg_sq[o : o + n].view_as(p)}
        lr = self.learning_rate()
        for group in opt.param_groups:
            group["lr"] = lr

    def sync_from_torch(self) -> None:
        """Pull loaded weights / optimizer state into the arena; refresh the bf16 shadows of student and teacher."""
        opt = self.alg.optimizer
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            if p.data.data_ptr() != self.flat[o : o + n].data_ptr():
                self.flat[o : o + n].copy_(p.data.reshape(-1))
                p.data = self.flat[o : o + n].view_as(p)
            st = opt.state.get(p)
            if st:
                self.exp_avg[o : o + n].copy_(st["exp_avg"].reshape(-1))
                self.exp_avg_sq[o : o + n].copy_(st["exp_avg_sq"].reshape(-1))
                self.step.fill_(int(float(st["step"])))
                opt.state[p] = {"step": st["step"], "exp_avg": self.exp_avg[o : o + n].view_as(p),
                                "exp_avg_sq": self.exp_avg_sq[o : o + n].view_as(p)}
        self.lr.fill_(float(opt.param_groups[0]["lr"]))
        self._refresh_shadows()

    # ---- data parallel ------------------------------------------------------------------------------------------------
    def broadcast_parameters(self) -> None:
        """Make every rank start from rank 0's student and teacher (parameters and normaliser buffers)."""
        if self.comm is not None:
            self.comm.broadcast_(self.flat, status=self.status)
            lo, hi = self.flat.data_ptr(), self.flat.data_ptr() + 4 * self.n_params
            tensors = [t for t in self.student.state_dict().values() if t.data_ptr() < lo or t.data_ptr() >= hi]
            tensors += list(self.teacher.state_dict().values())
            for t in tensors:
                self.comm.broadcast_(t, status=self.status)
            self._check_status()
        else:
            for model in (self.student, self.teacher):
                for t in model.state_dict().values():
                    torch.distributed.broadcast(t, src=0)
        self._refresh_shadows()


class RecurrentDistillationEngine(DistillationEngine):
    """Distillation with a GRU / LSTM student (see the module docstring for the window rule)."""

    @staticmethod
    def unsupported_reason(alg) -> str | None:
        return (rnn_model_reason("student", alg.student) or _teacher_reason(alg.teacher) or _common_reason(alg))

    def __init__(self, alg) -> None:
        st = alg.student
        self._init_common(alg, list(dict.fromkeys(chain(st.rnn.parameters(), st.mlp.parameters()))))
        # a training sequence is at most one window of steps over all environments, time-major
        self.L_max = min(self.GL, self.T)
        self.snet = _RecurrentNet(st, self.N, self.L_max, self.N, self.device, self.sm_count,
                                  alg.b200_cfg["rnn_fused_step"])
        self.snet.refresh_shadows()
        self.plan_s = self.snet.head
        self.head_s = self.plan_s.head_cols
        self._init_teacher()
        self._init_arena(self.N * self.L_max)
        seg = self.snet.reduce_segments(self.dhead_colsum, self.mse_blocks)
        self._init_reduce_and_adam(seg, self.snet.shadows())
        N, H, dev = self.N, self.snet.H, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        lstm = self.snet.lstm
        # state every epoch of the next update starts from (upstream's last_student_hidden_state; zero at first)
        self.h_last = torch.zeros(N, H, **f32)
        self.c_last = torch.zeros(N, H, **f32) if lstm else None
        # state after the last step of a sequence, masked by that step's dones
        self.carry_h = torch.zeros(N, H, **f32)
        self.carry_hbf = torch.zeros(N, H, dtype=torch.bfloat16, device=dev)
        self.carry_c = torch.zeros(N, H, **f32) if lstm else None

    def _refresh_shadows(self) -> None:
        self.snet.refresh_shadows()
        if self.tnet is not None:
            self.tnet.refresh_shadows()
        else:
            self.plan_t.refresh_shadows()

    # ---- rollout ------------------------------------------------------------------------------------------------------
    def _student_forward(self, x_rows: torch.Tensor) -> torch.Tensor:
        net = self.snet
        net.step(x_rows, x_rows.shape[1], self.status)
        head = net.head
        head.forward(net.h_bf, head.h_roll, self.N, head.out_roll, head.out_roll.shape[1], self.status)
        return head.out_roll

    def _reset_states(self, done_f: torch.Tensor) -> None:
        super()._reset_states(done_f)
        net = self.snet
        ext().rnn_mask(self.N, net.H, net.h, net.H, net.c, net.H, done_f, net.h, net.H, net.h_bf, net.H, net.c, net.H)

    # ---- update -------------------------------------------------------------------------------------------------------
    def _update_body(self) -> None:
        C = ext()
        N, T, GL = self.N, self.T, self.GL
        net, head = self.snet, self.snet.head
        H = net.H
        huber = self.alg.loss_type == "huber"
        self.loss_acc.zero_()
        carry = (self.carry_h, self.carry_hbf, self.carry_c)
        for _, t, L, first, train, apply in window_segments(self.E, T, GL):
            init = (self.h_last, self.c_last) if t == 0 else (self.carry_h, self.carry_c)
            x = self.x_s[t * N : (t + L) * N]
            rows = L * N
            used = C.mse_blocks(rows)
            if used < self.mse_blocks:  # fewer loss blocks: clear the output-bias partial rows they leave
                self.dhead_colsum[used:].zero_()
            net.forward_sequence(0, N, self.st_dones, head.out_train, head.out_train.shape[1], self.status, L=L, t0=t,
                                 time_major=True, x=x, init=init, carry=carry)
            # every step's loss is a mean over its N rows: the window's gradient is the sum of the step means'
            C.mse_grad(head.out_train, head.out_train.shape[1], self.targets[t * N : (t + L) * N], self.head_t, rows,
                       self.A, huber, head.d_head, head.d_head.shape[1], self.head_s, self.loss_partial,
                       self.dhead_colsum, self.loss_acc, self.loss_ticket, None, N)
            if train:
                net.backward_sequence(0, N, self.st_dones, self.status, L=L, t0=t, time_major=True, x=x)
                self._reduce(accumulate=not first)
                if apply:
                    self._adam()
        # the next update's epochs start from the state this one ended with, and the rollout continues from it
        C.rnn_mask(N, H, self.carry_h, H, self.carry_c, H, None, self.h_last, H, None, 0, self.c_last, H)
        C.rnn_mask(N, H, self.carry_h, H, self.carry_c, H, None, net.h, H, net.h_bf, H, net.c, H)
        self._normalizer_update("student", self.student, self.obs_s, self.total, self.Ds)


__all__ = ["DistillationEngine", "RecurrentDistillationEngine", "window_segments"]
