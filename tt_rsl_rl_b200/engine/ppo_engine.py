"""Fused CUDA engine of :class:`tt_rsl_rl_b200.algorithms.PPO`.

State lives on the device for the whole run: a flat fp32 parameter arena (the ``nn.Parameter``s of actor and critic
are views into it, so ``state_dict`` and checkpoints are unchanged), flat Adam moments (views installed into the
``torch.optim.Adam`` object on ``save``), bf16 weight shadows, the rollout arena ``[T * N, ...]`` and the minibatch
buffers. Per iteration:

* ``act`` / ``process_env_step``: observation concat + normalisation, actor and critic forward (tcgen05 GEMMs), the
  Gaussian head with Philox sampling, time-out bootstrap and storage writes;
* ``compute_returns``: critic forward on the last observation, GAE reverse scan, advantage normalisation;
* ``update``: for each of ``E x M`` minibatches: Feistel-permuted gather, forward of both models, fused PPO loss and
  output gradients, backward GEMMs, gradient reduction, and the fused (exchange +) clip + adaptive-LR + Adam kernel;
  then the observation normaliser update. From the second call on the whole update is one CUDA graph replay and the
  only host synchronisation is the read of the loss statistics at the end.

Extensions: with RND (``rsl_rl/extensions/rnd.py``) the target and predictor MLPs run on the same GEMMs, the intrinsic
reward is added on the device during the rollout and the predictor is a third parameter group of the fused optimizer
launch (its own learning rate, no clipping). With symmetry (``rsl_rl/extensions/symmetry.py``) the augmentation
function is probed once as per-copy signed permutations; the gather kernel writes the mirrored observation copies and
the loss kernel mirrors the actions and adds the mirror-loss gradient.

Semantics follow ``rsl_rl/algorithms/ppo.py`` (see the kernels' comments for the exact rules). The random number
streams differ from PyTorch's (Philox in-kernel sampling, Feistel permutation instead of ``torch.randperm``).
"""

from __future__ import annotations

from itertools import chain

import torch

from ..modules import GaussianDistribution, HeteroscedasticGaussianDistribution
from ..ops import ext
from ..utils.timer import HostTransfers
from .base import EngineBase, elu_mlp_reason
from .mlp_plan import MLPPlan
from .rnd_part import RndPart, rnd_reason

_GROUP_ACTOR = 0
_GROUP_CRITIC = 1
_GROUP_RND = 2
_TAIL = 5  # exchanged statistics after the parameters: surrogate, value, entropy, kl, symmetry (minibatch means)
_MAX_COPIES = 8


def _padded_rows(rows: int, dim: int, device) -> torch.Tensor:
    """A [rows, dim] fp32 view of a zero buffer whose row pitch is dim rounded up to 4 floats (16 bytes)."""
    return torch.zeros(rows, (dim + 3) // 4 * 4, dtype=torch.float32, device=device)[:, :dim]


def _model_maps(obs_maps: dict, groups: list[str], K: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Concatenate per-group signed permutations into the model's input columns: (perm [K, D] int32, sign [K, D])."""
    perms, signs, off = [], [], 0
    for g in groups:
        perm, sign = obs_maps[g]
        if perm.shape[0] != K:
            raise ValueError("symmetry: every observation group needs the same number of copies")
        perms.append(perm + off)
        signs.append(sign)
        off += perm.shape[1]
    return (torch.cat(perms, 1).to(device=device, dtype=torch.int32).contiguous(),
            torch.cat(signs, 1).to(device=device, dtype=torch.float32).contiguous())


class PPOEngine(EngineBase):
    # ---- capability checks ------------------------------------------------------------------------------------------
    @staticmethod
    def supports_models(actor, critic, alg_cfg: dict) -> str | None:
        from ..models import CNNModel, MLPModel

        for name, m in (("actor", actor), ("critic", critic)):
            if type(m) is not MLPModel:
                if isinstance(m, CNNModel):
                    return f"{name} is a CNNModel"
                return f"{name} type {type(m).__name__} is not fused"
            reason = elu_mlp_reason(m)
            if reason:
                return f"{name}: {reason}"
            if m.obs_dim > 1024:
                return f"{name} observation width {m.obs_dim} too large"
        dist = actor.distribution
        if not isinstance(dist, (GaussianDistribution, HeteroscedasticGaussianDistribution)):
            return "actor distribution is not Gaussian"
        if dist.output_dim > 32:
            return "more than 32 actions"
        if critic.distribution is not None:
            return "critic has a distribution"
        if critic.mlp.linears[-1].out_features != 1:
            return "critic output is not scalar"
        rnd_cfg = alg_cfg.get("rnd_cfg")
        if isinstance(rnd_cfg, dict):
            if str(rnd_cfg.get("activation", "elu")).lower() != "elu":
                return "RND activation is not fused (ELU only)"
        if str(alg_cfg.get("optimizer", "adam")).lower() != "adam":
            return "only Adam is fused"
        return None

    @staticmethod
    def unsupported_reason(alg) -> str | None:
        cfg = {
            "normalize_advantage_per_mini_batch": alg.normalize_advantage_per_mini_batch,
            "optimizer": getattr(alg, "optimizer_name", "adam"),
        }
        reason = PPOEngine.supports_models(alg.actor, alg.critic, cfg)
        if reason is not None:
            return reason
        if alg.rnd is not None:
            reason = rnd_reason(alg.rnd)
            if reason is not None:
                return reason
        if alg.symmetry is not None:
            template = getattr(alg, "_obs_template", None)
            if template is None:
                return "symmetry needs the observation template to probe the augmentation"
            A = alg.actor.distribution.output_dim
            maps = alg.symmetry.probe_signed_permutations(template, A)
            if maps is None:
                return "symmetry augmentation is not a per-copy signed permutation"
            obs_maps, act_maps = maps
            K = int(act_maps[0].shape[0])
            if not 2 <= K <= _MAX_COPIES:
                return f"symmetry with {K} copies"
            groups = set(alg.actor.obs_groups) | set(alg.critic.obs_groups)
            if any(obs_maps[g][0].shape[0] != K for g in groups):
                return "symmetry copies differ between observation groups and actions"
            alg._symmetry_maps = maps
        return None

    # ---- construction -------------------------------------------------------------------------------------------------
    def __init__(self, alg, num_steps_per_env: int, num_envs: int, obs_template) -> None:
        self.alg = alg
        self.device = torch.device(alg.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.T = num_steps_per_env
        self.N = num_envs
        self.total = self.T * self.N
        self.M = alg.num_mini_batches
        self.E = alg.num_learning_epochs
        if not 1 <= self.M <= self.total:
            raise ValueError("num_mini_batches must be between 1 and the rollout batch size.")
        self.B_max = max((i + 1) * self.total // self.M - i * self.total // self.M for i in range(self.M))
        props = torch.cuda.get_device_properties(self.device)
        self.sm_count = props.multi_processor_count
        self.actor = alg.actor
        self.critic = alg.critic
        dist = self.actor.distribution
        self.hetero = isinstance(dist, HeteroscedasticGaussianDistribution)
        self.log_std = dist.std_type == "log"
        self.A = dist.output_dim
        self.std_range = dist.std_range
        self.log_std_range = dist.log_std_range
        dev = self.device
        f32 = dict(dtype=torch.float32, device=dev)

        # observation layout
        self.groups_a = list(self.actor.obs_groups)
        self.groups_c = list(self.critic.obs_groups)
        self.Da = self.actor.obs_dim
        self.Dc = self.critic.obs_dim
        self.shared_obs = self.groups_a == self.groups_c

        # ---- symmetry: K copies of every minibatch row (copy 0 = the sample) ----
        self.sym = alg.symmetry
        self.K, self.aug, self.mirror_coef = 1, False, 0.0
        self.perm_a = self.sign_a = self.perm_c = self.sign_c = self.act_perm = self.act_sign = None
        if self.sym is not None:
            obs_maps, act_maps = alg._symmetry_maps
            self.K = int(act_maps[0].shape[0])
            self.aug = bool(self.sym.use_data_augmentation)
            self.mirror_coef = float(self.sym.mirror_loss_coeff) if self.sym.use_mirror_loss else 0.0
            self.perm_a, self.sign_a = _model_maps(obs_maps, self.groups_a, self.K, dev)
            self.perm_c, self.sign_c = _model_maps(obs_maps, self.groups_c, self.K, dev)
            self.act_perm = act_maps[0].to(device=dev, dtype=torch.int32).contiguous()
            self.act_sign = act_maps[1].to(device=dev, dtype=torch.float32).contiguous()
        self.rows_a_max = self.K * self.B_max
        self.rows_c_max = self.rows_a_max if self.aug else self.B_max
        self.rnd = alg.rnd

        # ---- flat parameter arena (views installed into the nn.Parameters) ----
        self.params = list(dict.fromkeys(chain(self.actor.parameters(), self.critic.parameters())))
        actor_ids = {id(p) for p in self.actor.parameters()}
        self.param_group = [_GROUP_ACTOR if id(p) in actor_ids else _GROUP_CRITIC for p in self.params]
        if self.rnd is not None:
            rnd_params = list(self.rnd.predictor.parameters())
            self.params += rnd_params
            self.param_group += [_GROUP_RND] * len(rnd_params)
        self.offsets = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += p.numel()
        self.n_params = off
        self.flat = torch.zeros(self.n_params, **f32)
        for p, o in zip(self.params, self.offsets):
            self.flat[o : o + p.numel()].copy_(p.data.reshape(-1))
            p.data = self.flat[o : o + p.numel()].view_as(p)
        n_ex = (self.n_params + _TAIL + 3) // 4 * 4  # exchanged floats: parameters + statistics, float4 granules
        self.n_ex = n_ex
        n_actor = sum(p.numel() for p, g in zip(self.params, self.param_group) if g == _GROUP_ACTOR)
        n_ac = sum(p.numel() for p, g in zip(self.params, self.param_group) if g != _GROUP_RND)
        if self.param_group != sorted(self.param_group):
            raise RuntimeError("fused engine: actor parameters must precede critic parameters")
        self.group_ranges = [0, n_actor, n_actor, n_ac]
        if self.rnd is not None:
            self.group_ranges += [n_ac, self.n_params]
        self.exp_avg = torch.zeros(self.n_params, **f32)
        self.exp_avg_sq = torch.zeros(self.n_params, **f32)
        # ---- data parallel: symmetric send buffers shared with the peers (CUDA IPC) ----
        self.world = alg.gpu_world_size
        self.rank = alg.gpu_global_rank
        self.timeout_ns = int(alg.b200_cfg["comm_timeout_ms"] * 1e6)
        self.comm = None
        self._peer_reduced = None  # set for the two-shot exchange
        self._kl_offset = self.n_params + 3  # index of the KL statistic in the exchanged vector
        if self.world > 1:
            from ..parallel import PeerExchange

            big = max((t.numel() for t in self.rnd.state_dict().values()), default=0) if self.rnd is not None else 0
            dmax = max(self.Da, self.Dc, self.rnd.num_states if self.rnd is not None else 0)
            small = max(4 * self.n_params, 4 * big, 8 * (2 + 2 * dmax), 4096)
            self.comm = PeerExchange.create(n_ex, small, rank=self.rank, world=self.world, device=dev,
                                            timeout_ms=alg.b200_cfg["comm_timeout_ms"])
            from ..algorithms.ppo import use_two_shot

            # two-shot exchange: the ranks' reduced buffers; the KL statistic is read from its owner's shard
            if use_two_shot(alg.b200_cfg, self.world):
                self._peer_reduced = self.comm.peer_reduced

            self.send = self.comm.send
        else:
            buf = torch.zeros(n_ex, **f32)
            self.send = [buf, buf]
        self.grads = torch.zeros(n_ex, **f32)
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
        self.perm_key = torch.zeros(1, dtype=torch.int32, device=dev)
        self.seed = int(torch.initial_seed() % (2**62))
        self.half_bits = ext().feistel_half_bits(self.total)
        if self.total >= 2**31:
            raise ValueError("rollout batch too large for the fused engine")

        # ---- MLP plans ----
        self.plan_a = MLPPlan(self.actor.mlp, self.Da, self.N, self.rows_a_max, dev, self.sm_count)
        self.plan_c = MLPPlan(self.critic.mlp, self.Dc, self.N, self.rows_c_max, dev, self.sm_count)
        self.head_cols = self.plan_a.head_cols
        self.plans = [self.plan_a, self.plan_c]
        self.rnd_part = None
        if self.rnd is not None:
            self.rnd_part = RndPart(self, self.rnd, self.N, self.T, self.B_max, dev, self.sm_count)
            self.Dr = self.rnd_part.Dr
            self.groups_r = self.rnd_part.groups
            self.plan_rp = self.rnd_part.plan_p
            self.plans += self.rnd_part.plans
        for plan in self.plans:
            plan.refresh_shadows()

        # ---- rollout arena ----
        T, N, A = self.T, self.N, self.A
        # observation arenas: rows padded to 16 bytes so the minibatch gather reads them with 16-byte loads
        self.obs_a = _padded_rows(T * N, self.Da, dev)
        self.obs_c = self.obs_a if self.shared_obs else _padded_rows(T * N, self.Dc, dev)
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
        self.gae_partial = torch.zeros(2 * ext().gae_blocks(N), dtype=torch.float64, device=dev)
        self.t = 0
        self.intrinsic_for_logger = None
        if self.rnd is not None:
            if self.groups_r == self.groups_a:
                self.obs_r = self.obs_a
            elif self.groups_r == self.groups_c:
                self.obs_r = self.obs_c
            else:
                self.obs_r = _padded_rows(T * N, self.Dr, dev)
            self.intrinsic_for_logger = self.rnd_part.intrinsic
            alg.intrinsic_rewards = self.rnd_part.intrinsic

        # ---- minibatch buffers ----
        B = self.B_max
        self.idx = torch.zeros(B, dtype=torch.int32, device=dev)
        self.value_train = torch.zeros(self.rows_c_max, 1, **f32)
        self.d_value = self.plan_c.d_head  # gradient of the scalar value head, [rows, 8] bf16 (7 zero padding columns)
        self.loss_blocks = ext().ppo_loss_blocks(self.rows_a_max)
        self.stats_partial = torch.zeros(self.loss_blocks, _TAIL, **f32)
        self.dhead_colsum = torch.zeros(self.loss_blocks, self.head_cols, **f32)
        self.dvalue_colsum = torch.zeros(self.loss_blocks, 1, **f32)
        self.dstd_partial = torch.zeros(self.loss_blocks, A, **f32)
        self.loss_acc = torch.zeros(_TAIL, **f32)
        # normalize_advantage_per_mini_batch: the minibatch's advantages, normalised, replace the stored ones
        self.adv_per_mb = bool(alg.normalize_advantage_per_mini_batch)
        self.adv_mb = torch.zeros(B, **f32) if self.adv_per_mb else None
        self.adv_mb_partial = (torch.zeros(2 * ext().adv_gather_blocks(B), dtype=torch.float64, device=dev)
                               if self.adv_per_mb else None)

        # ---- gradient reduction plan (flat order = optimizer order) ----
        seg = {}
        seg.update(self.plan_a.reduce_segments(self.dhead_colsum, self.loss_blocks))
        seg.update(self.plan_c.reduce_segments(self.dvalue_colsum, self.loss_blocks))
        if self.rnd is not None:
            seg.update(self.rnd_part.reduce_segments())
        if not self.hetero:
            std_p = dist.std_param if dist.std_type == "scalar" else dist.log_std_param
            seg[id(std_p)] = (self.dstd_partial, self.loss_blocks, A)
        srcs, parts, ns, offs = [], [], [], []
        for p, o in zip(self.params, self.offsets):
            if id(p) not in seg:
                raise RuntimeError("fused engine: parameter without a gradient source")
            buf, nparts, n = seg[id(p)]
            srcs.append(buf)
            parts.append(nparts)
            ns.append(n)
            offs.append(o)
        srcs.append(self.stats_partial)
        parts.append(self.loss_blocks)
        ns.append(_TAIL)
        offs.append(self.n_params)
        self.reduce_plan, self.reduce_nseg, self.reduce_chunks = ext().make_reduce_plan(srcs, parts, ns, offs)

        # ---- Adam plan ----
        shadows = {}
        for plan in self.plans:
            if not plan.train or not plan.grads:
                continue
            for lin, wb in zip(plan.linears, plan.w_bf16):
                shadows[id(lin.weight)] = wb
        t_off, t_num, t_grp, t_rows, t_cols, t_sh, t_ld = [], [], [], [], [], [], []
        for p, o, g in zip(self.params, self.offsets, self.param_group):
            t_off.append(o)
            t_num.append(p.numel())
            t_grp.append(g)
            sh = shadows.get(id(p))
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
        self.adam_tensors, self.adam_chunks, self.adam_nchunks = ext().make_adam_plan(
            t_off, t_num, t_grp, t_rows, t_cols, t_sh, t_ld, self.flat
        )
        self.adam_grid = ext().adam_grid(self.device.index)
        self.norm_partial = torch.zeros(self.adam_grid * 4, **f32)
        self.out_norms = torch.zeros(4, **f32)
        opt = alg.optimizer
        group0 = opt.param_groups[0]
        b1, b2 = group0.get("betas", (0.9, 0.999))
        self.betas = (float(b1), float(b2))
        self.adam_eps = float(group0.get("eps", 1e-8))
        if float(group0.get("weight_decay", 0.0)) != 0.0 or group0.get("amsgrad", False):
            raise ValueError("fused Adam supports weight_decay=0 and amsgrad=False")
        ng = 3 if self.rnd is not None else 2
        self.adam_max_norm = [alg.max_grad_norm, alg.max_grad_norm] + [0.0] * (ng - 2)
        self.adam_beta1 = [self.betas[0]] * 2
        self.adam_beta2 = [self.betas[1]] * 2
        self.adam_eps_g = [self.adam_eps] * 2
        self.adam_lr_index = [0, 0]
        if self.rnd is not None:
            rb1, rb2, reps = self.rnd_part.adam_hparams()
            self.adam_beta1.append(rb1)
            self.adam_beta2.append(rb2)
            self.adam_eps_g.append(reps)
            self.adam_lr_index.append(2)

        # ---- normaliser statistics scratch ----
        self._alloc_norm_scratch("actor", self.total, self.Da)
        self._alloc_norm_scratch("critic", self.total, self.Dc)
        self.use_graphs = bool(alg.b200_cfg["graphs"])
        self._update_graph = None
        self._updates_done = 0
        self.perm_override: torch.Tensor | None = None  # int32 [T*N]: explicit sample order (tests, reproducibility)
        self._init_base()
        self._init_streams(alg.b200_cfg)

    # ---- learning rate -----------------------------------------------------------------------------------------------
    def learning_rate(self) -> float:
        return float(HostTransfers.read(self.lr[0:1], "learning_rate")[0])

    def set_learning_rate(self, value: float) -> None:
        self.lr[0].fill_(value)

    def action_std(self) -> torch.Tensor:
        """Current policy std (for logging): the clamped parameter, or the mean per-row std of the last rollout."""
        dist = self.actor.distribution
        if self.hetero:
            return self.st_std.mean(dim=0)
        return dist.current_std().detach()

    # ---- rollout ------------------------------------------------------------------------------------------------------
    def act(self, obs) -> torch.Tensor:
        if self.t >= self.T:
            raise OverflowError("Rollout buffer overflow! You should call clear() before adding new transitions.")
        N, t = self.N, self.t
        rows = slice(t * N, (t + 1) * N)
        C = ext()
        if self.rnd is not None and t == 0 and not torch.cuda.is_current_stream_capturing():
            self.rnd_part.prepare()
        if self.rnd is not None and self.obs_r is not self.obs_a and self.obs_r is not self.obs_c:
            # the RND state groups are stored on their own (normalised copy goes to a scratch buffer)
            C.prep_obs(self._group_tensors(obs, self.groups_r), self.obs_r[rows], self.obs_r.stride(0),
                       self.plan_rp.x_roll,
                       self.plan_rp.x_roll.shape[1], None, None, 0.0)
        mean_a, std_a, eps_a = self._norm_tensors(self.actor)
        C.prep_obs(self._group_tensors(obs, self.groups_a), self.obs_a[rows], self.obs_a.stride(0), self.plan_a.x_roll,
                   self.plan_a.x_roll.shape[1], mean_a, std_a, eps_a)
        mean_c, std_c, eps_c = self._norm_tensors(self.critic)
        store_c = None if self.shared_obs else self.obs_c[rows]
        C.prep_obs(self._group_tensors(obs, self.groups_c), store_c, self.obs_c.stride(0), self.plan_c.x_roll,
                   self.plan_c.x_roll.shape[1], mean_c, std_c, eps_c)
        pa, pc = self.plan_a, self.plan_c
        dist = self.actor.distribution
        std_param = None if self.hetero else (dist.std_param if dist.std_type == "scalar" else dist.log_std_param)

        def actor_step():
            pa.forward(pa.x_roll, pa.h_roll, N, pa.out_roll, pa.out_roll.shape[1], self.status)
            C.gaussian_sample(pa.out_roll, pa.out_roll.shape[1], N, self.A, self.hetero, self.log_std,
                              None if std_param is None else std_param.data, self.std_range[0], self.std_range[1],
                              self.log_std_range[0], self.log_std_range[1], self.seed, self.rng_counter,
                              self.rng_ticket, self.st_actions[rows], self.st_mean[rows], self.st_std[rows],
                              self.st_logp[rows], self.actions_out)

        # actor (with sampling) and critic are independent: two streams, joined before the actions are returned
        self._in_parallel(actor_step,
                          lambda: pc.forward(pc.x_roll, pc.h_roll, N, self.st_values[rows].view(N, 1), 1, self.status))
        return self.actions_out

    def process_env_step(self, obs, rewards, dones, extras) -> None:
        N, t = self.N, self.t
        rows = slice(t * N, (t + 1) * N)
        timeouts = extras.get("time_outs") if isinstance(extras, dict) else None
        if timeouts is not None:
            timeouts = timeouts.to(self.device).reshape(-1)
        intrinsic = None
        if self.rnd is not None:
            intrinsic = self.rnd_part.intrinsic_reward(self, obs, t)
        ext().process_step(rewards.reshape(-1).float(), intrinsic, dones.reshape(-1), timeouts, self.st_values[rows],
                           self.alg.gamma, self.st_rewards[rows], self.st_dones[rows], self.nonfinite)
        self.t += 1

    def _before_replay(self) -> None:
        if self.rnd is not None:
            self.rnd_part.prepare()

    def compute_returns(self, obs) -> None:
        C = ext()
        mean_c, std_c, eps_c = self._norm_tensors(self.critic)
        pc = self.plan_c
        C.prep_obs(self._group_tensors(obs, self.groups_c), None, self.Dc, pc.x_roll, pc.x_roll.shape[1], mean_c,
                   std_c, eps_c)
        pc.forward(pc.x_roll, pc.h_roll, self.N, self.last_values.view(self.N, 1), 1, self.status)
        C.gae(self.st_rewards, self.st_dones, self.st_values, self.last_values, self.st_returns, self.st_adv, self.T,
              self.N, self.alg.gamma, self.alg.lam, self.gae_partial)
        if self.total > 1 and not self.adv_per_mb:
            C.adv_normalize(self.st_adv, self.gae_partial, ext().gae_blocks(self.N))
        self.t = 0

    # ---- update -------------------------------------------------------------------------------------------------------
    def _zero_partial_tails(self, B: int) -> None:
        """A minibatch shorter than the largest one launches fewer loss blocks: clear the unused partial rows."""
        C = ext()
        used = C.ppo_loss_blocks(self.K * B)
        if used < self.loss_blocks:
            for buf in (self.stats_partial, self.dhead_colsum, self.dvalue_colsum, self.dstd_partial):
                buf[used:].zero_()
        if self.rnd is not None:
            self.rnd_part.zero_tails(B)

    def _minibatch_advantages(self, idx: torch.Tensor, n: int):
        """normalize_advantage_per_mini_batch: (adv[idx] - mean) / (std + 1e-8) over the minibatch, else None."""
        if not self.adv_per_mb or n <= 1:
            return None
        C = ext()
        C.adv_gather_stats(self.st_adv, idx, n, self.adv_mb, self.adv_mb_partial, self.status)
        C.adv_normalize(self.adv_mb[:n], self.adv_mb_partial, C.adv_gather_blocks(n))
        return self.adv_mb

    def _minibatch(self, i: int) -> None:
        C = ext()
        start = i * self.total // self.M
        B = (i + 1) * self.total // self.M - start
        if B < self.B_max:
            self._zero_partial_tails(B)
        rows_a = self.K * B
        rows_c = rows_a if self.aug else B
        pa, pc = self.plan_a, self.plan_c
        mean_a, std_a, eps_a = self._norm_tensors(self.actor)
        mean_c, std_c, eps_c = self._norm_tensors(self.critic)
        eps_all = {e for m, e in ((mean_a, eps_a), (mean_c, eps_c)) if m is not None}
        obs_l, mean_l, std_l = [self.obs_a, self.obs_c], [mean_a, mean_c], [std_a, std_c]
        x_l, ld_l, rows_l = [pa.x_train, pc.x_train], [pa.x_train.shape[1], pc.x_train.shape[1]], [rows_a, rows_c]
        perm_l = [self.perm_a, self.perm_c if self.aug else None]
        sign_l = [self.sign_a, self.sign_c if self.aug else None]
        if self.rnd is not None:
            mean_r, std_r, eps_r = self._norm_views(self.rnd.state_normalizer)
            if mean_r is not None:
                eps_all.add(eps_r)
            obs_l.append(self.obs_r)
            mean_l.append(mean_r)
            std_l.append(std_r)
            x_l.append(self.plan_rp.x_train)
            ld_l.append(self.plan_rp.x_train.shape[1])
            rows_l.append(B)
            perm_l.append(None)
            sign_l.append(None)
        if len(eps_all) > 1:
            raise ValueError("all fused observation normalisers must share eps")
        eps = eps_all.pop() if eps_all else 0.0
        idx_in = None if self.perm_override is None else self.perm_override[start : start + B]
        C.gather_minibatch(B, start, self.total, self.perm_key, self.half_bits, idx_in, self.idx, obs_l, mean_l, std_l,
                           eps, x_l, ld_l, self.status, self.K, rows_l, perm_l, sign_l)
        adv_override = self._minibatch_advantages(self.idx, B)
        self._in_parallel(
            lambda: pa.forward(pa.x_train, pa.h_train, rows_a, pa.out_train, pa.out_train.shape[1], self.status),
            lambda: pc.forward(pc.x_train, pc.h_train, rows_c, self.value_train, 1, self.status))
        dist = self.actor.distribution
        std_param = None if self.hetero else (dist.std_param if dist.std_type == "scalar" else dist.log_std_param)
        alg = self.alg
        C.ppo_loss(B, self.A, self.hetero, self.log_std, pa.out_train, pa.out_train.shape[1], self.value_train, 1,
                   None if std_param is None else std_param.data, self.std_range[0], self.std_range[1],
                   self.log_std_range[0], self.log_std_range[1], self.idx, self.st_actions, self.st_mean, self.st_std,
                   self.st_logp, self.st_adv, self.st_returns, self.st_values, adv_override, alg.clip_param,
                   alg.value_loss_coef, alg.entropy_coef, alg.use_clipped_value_loss, pa.d_head, pa.d_head.shape[1],
                   self.d_value, self.d_value.shape[1], self.stats_partial, self.dhead_colsum, self.dvalue_colsum,
                   None if self.hetero else self.dstd_partial, self.K, self.aug, self.act_perm, self.act_sign,
                   self.mirror_coef, self.status)
        self._in_parallel(lambda: pa.backward(rows_a, self.status), lambda: pc.backward(rows_c, self.status))
        if self.rnd is not None:
            self.rnd_part.train(B, self.status)
        C.reduce_segments(self.reduce_plan, self.reduce_nseg, self.reduce_chunks, self.send[0], self.send[1],
                          self.epoch, False)
        adaptive = alg.desired_kl is not None and alg.schedule == "adaptive"
        kl = self.grads[self.n_params + 3 : self.n_params + 4]
        peers = self.comm.peer_send if self.comm is not None else None
        flags = self.comm.peer_flags if self.comm is not None else None
        C.adam_step(self.flat, self.send[0], self.send[1], self.grads, self.exp_avg, self.exp_avg_sq,
                    self.adam_tensors, self.adam_chunks, self.adam_nchunks, self.adam_max_norm, self.adam_beta1,
                    self.adam_beta2, self.adam_eps_g, self.adam_lr_index, self.lr, None, self.step, adaptive, kl,
                    float(alg.desired_kl or 0.0), 1e-5, 1e-2, self.world, self.rank, peers, flags, self.epoch,
                    self.timeout_ns, self.norm_partial, self.barrier, self.status, self.out_norms, self.adam_grid,
                    self.group_ranges, self.n_ex, self._peer_reduced, self._kl_offset)
        self.loss_acc.add_(self.grads[self.n_params : self.n_params + _TAIL])

    def _normalizer_updates(self) -> None:
        self._normalizer_update("actor", self.actor, self.obs_a, self.total, self.Da)
        self._normalizer_update("critic", self.critic, self.obs_c, self.total, self.Dc)
        if self.rnd is not None:
            self.rnd_part.normalizer_update(self, self.obs_r, self.total)

    def _update_body(self) -> None:
        ext().counter_add(self.perm_key, 1)
        self.loss_acc.zero_()
        if self.rnd is not None:
            self.rnd_part.loss_acc.zero_()
        for _ in range(self.E):
            for i in range(self.M):
                self._minibatch(i)
        self._normalizer_updates()

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
        if self.sym is not None:
            out["symmetry"] = stats[4]
        return out

    # ---- rollout import (tests / external collectors) -------------------------------------------------------------------
    def load_rollout(self, storage) -> None:
        """Copy a filled :class:`RolloutStorage` (``[T, N, ...]`` tensors, returns/advantages computed) into the arena."""
        T, N = self.T, self.N
        obs = storage.observations.flatten(0, 1)
        self.obs_a.copy_(torch.cat([obs[g] for g in self.groups_a], dim=-1))
        if not self.shared_obs:
            self.obs_c.copy_(torch.cat([obs[g] for g in self.groups_c], dim=-1))
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
            n = p.numel()
            if steps[g] == 0:
                continue
            self._optimizer_of(g).state[p] = {
                "step": torch.tensor(float(steps[g])),
                "exp_avg": self.exp_avg[o : o + n].view_as(p),
                "exp_avg_sq": self.exp_avg_sq[o : o + n].view_as(p),
            }
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
            self.lr[2] = float(self.rnd.optimizer.param_groups[0]["lr"])
        for plan in self.plans:
            plan.refresh_shadows()

    # ---- data parallel ------------------------------------------------------------------------------------------------
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
            models = [self.actor, self.critic] + ([self.rnd] if self.rnd is not None else [])
            for model in models:
                for t in model.state_dict().values():
                    torch.distributed.broadcast(t, src=0)
        for plan in self.plans:
            plan.refresh_shadows()


__all__ = ["PPOEngine"]
