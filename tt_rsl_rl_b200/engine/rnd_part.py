"""Device part of Random Network Distillation shared by the fused PPO engines.

Semantics: ``rsl_rl/extensions/rnd.py`` (``get_intrinsic_reward``, ``compute_loss``, the weight schedule) and the
reward normaliser of ``rsl_rl/modules/normalization.py`` (``EmpiricalDiscountedVariationNormalization``). On the
device: the frozen target and the trained predictor MLPs run on the tcgen05 GEMMs; the intrinsic reward of every
post-step observation is ``weight * || target(s) - predictor(s) ||`` (optionally divided by the running std of its
per-environment discounted sum); the predictor's MSE step writes its output gradient and bias column sums for the
engine's segment reduction, so its gradient joins the fused optimizer launch as a parameter group of its own.
"""

from __future__ import annotations

import torch

from ..ops import ext
from .base import elu_stack_reason
from .mlp_plan import MLPPlan


def rnd_reason(rnd) -> str | None:
    """None if the RND module's networks and sizes are covered by the fused kernels, else the reason."""
    for name in ("predictor", "target"):
        reason = elu_stack_reason(getattr(rnd, name))
        if reason:
            return f"RND {name}: {reason}"
    if rnd.num_outputs > 64 or rnd.num_states > 1024:
        return "RND network too wide"
    return None


class RndPart:
    """RND plans and buffers of one engine: ``train_rows`` rows per predictor training step, ``N`` environments."""

    def __init__(self, engine, rnd, N: int, T: int, train_rows: int, device, sm_count: int) -> None:
        self.rnd = rnd
        self.N, self.T = N, T
        self.Dr, self.R = rnd.num_states, rnd.num_outputs
        self.groups = list(rnd.obs_groups["rnd_state"])
        self.plan_p = MLPPlan(rnd.predictor, self.Dr, N, train_rows, device, sm_count)
        self.plan_t = MLPPlan(rnd.target, self.Dr, N, train_rows, device, sm_count, grads=False)
        f32 = dict(dtype=torch.float32, device=device)
        self.intrinsic = torch.zeros(N, **f32)
        self.w = torch.zeros(T, **f32)  # per-step intrinsic weight of the current rollout
        self.tout_roll = torch.zeros(N, self.R, **f32)
        self.pout_roll = torch.zeros(N, self.R, **f32)
        self.tout_train = torch.zeros(train_rows, self.R, **f32)
        self.blocks = ext().mse_blocks(train_rows)
        self.loss_partial = torch.zeros(self.blocks, **f32)
        self.colsum = torch.zeros(self.blocks, self.R, **f32)
        self.loss_acc = torch.zeros(1, **f32)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=device)
        # reward normalisation: per-environment discounted sum of the raw intrinsic reward and its running std
        self.reward_norm = bool(rnd.reward_normalization)
        self.disc = torch.zeros(N, **f32) if self.reward_norm else None
        engine._alloc_norm_scratch("rnd", T * N, self.Dr)
        if self.reward_norm:
            engine._alloc_norm_scratch("rnd_reward", N, 1)

    # ---- structure ----------------------------------------------------------------------------------------------------
    @property
    def plans(self) -> list[MLPPlan]:
        return [self.plan_p, self.plan_t]

    def parameters(self) -> list[torch.nn.Parameter]:
        return list(self.rnd.predictor.parameters())

    def reduce_segments(self) -> dict[int, tuple]:
        return self.plan_p.reduce_segments(self.colsum, self.blocks)

    def adam_hparams(self) -> tuple[float, float, float]:
        """(beta1, beta2, eps) of the predictor's optimizer; the fused step has no weight decay / amsgrad."""
        g = self.rnd.optimizer.param_groups[0]
        b1, b2 = g.get("betas", (0.9, 0.999))
        if float(g.get("weight_decay", 0.0)) != 0.0 or g.get("amsgrad", False):
            raise ValueError("fused Adam supports weight_decay=0 and amsgrad=False")
        return float(b1), float(b2), float(g.get("eps", 1e-8))

    def learning_rate(self) -> float:
        return float(self.rnd.optimizer.param_groups[0]["lr"])

    def broadcast_modules(self) -> list:
        """Modules whose state rank 0 broadcasts besides the flat parameter arena (the predictor's are in it)."""
        return [self.rnd.target, self.rnd.state_normalizer, self.rnd.reward_normalizer]

    # ---- rollout ------------------------------------------------------------------------------------------------------
    def prepare(self) -> None:
        """Advance the host-side RND step counter by one rollout and upload the per-step intrinsic weights."""
        r = self.rnd
        weights = []
        for _ in range(self.T):
            r.update_counter += 1
            r.weight = r.current_weight(r.update_counter)
            weights.append(float(r.weight))
        self.w.copy_(torch.tensor(weights, dtype=torch.float32))

    def intrinsic_reward(self, engine, obs, t: int) -> torch.Tensor:
        """Intrinsic reward of the post-step observations of step ``t`` into ``self.intrinsic``."""
        C = ext()
        pr, pt = self.plan_p, self.plan_t
        mean_r, std_r, eps_r = engine._norm_views(self.rnd.state_normalizer)
        C.prep_obs(engine._group_tensors(obs, self.groups), None, self.Dr, pr.x_roll, pr.x_roll.shape[1], mean_r,
                   std_r, eps_r)
        pt.forward(pr.x_roll, pt.h_roll, self.N, self.tout_roll, self.R, engine.status)
        pr.forward(pr.x_roll, pr.h_roll, self.N, self.pout_roll, self.R, engine.status)
        w = self.w[t : t + 1]
        if not self.reward_norm:
            C.rnd_intrinsic(self.tout_roll, self.R, self.pout_roll, self.R, self.N, self.R, w, self.intrinsic, None,
                            0.0)
            return self.intrinsic
        # normalised: raw distance, discounted sum, running std of the sum (global over ranks), then weight / std
        rn = self.rnd.reward_normalizer
        C.rnd_intrinsic(self.tout_roll, self.R, self.pout_roll, self.R, self.N, self.R, w, self.intrinsic, self.disc,
                        rn.disc_avg.gamma)
        engine._norm_module_update("rnd_reward", rn.emp_norm, rn.training, self.disc.view(self.N, 1), self.N, 1)
        C.rnd_reward_scale(self.intrinsic, self.N, w, rn.emp_norm._std.view(-1))
        return self.intrinsic

    # ---- update -------------------------------------------------------------------------------------------------------
    def zero_tails(self, rows: int) -> None:
        """A step over fewer rows than the largest launches fewer loss blocks: clear the unused partial rows."""
        used = ext().mse_blocks(rows)
        if used < self.blocks:
            self.loss_partial[used:].zero_()
            self.colsum[used:].zero_()

    def train(self, rows: int, status, last_weight: torch.Tensor | None = None) -> None:
        """Predictor MSE step on the normalised rows already in ``plan_p.x_train``: target and predictor forward, the
        loss gradient (the last row weighted by ``last_weight`` when given) and the predictor backward."""
        C = ext()
        pr, pt = self.plan_p, self.plan_t
        pt.forward(pr.x_train, pt.h_train, rows, self.tout_train, self.R, status)
        pr.forward(pr.x_train, pr.h_train, rows, pr.out_train, self.R, status)
        C.mse_grad(pr.out_train, self.R, self.tout_train, self.R, rows, self.R, False, pr.d_head, pr.d_head.shape[1],
                   self.R, self.loss_partial, self.colsum, self.loss_acc, self.ticket, last_weight, 0)
        pr.backward(rows, status)

    def normalizer_update(self, engine, obs_r: torch.Tensor, total: int) -> None:
        engine._norm_module_update("rnd", self.rnd.state_normalizer, self.rnd.state_normalization, obs_r, total,
                                   self.Dr)


__all__ = ["RndPart", "rnd_reason"]
