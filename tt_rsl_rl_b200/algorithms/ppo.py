"""Proximal Policy Optimization with rsl_rl's public interface and semantics (``rsl_rl/algorithms/ppo.py``).

Two execution paths share this class:

* **CUDA (default on a CUDA device for MLP actor/critic with ELU hidden layers and a Gaussian or heteroscedastic
  Gaussian policy):** :class:`tt_rsl_rl_b200.engine.PPOEngine` owns device-resident rollout buffers and runs the act
  step, GAE, minibatch gather, fused forward/loss/backward (tcgen05 GEMMs) and the fused gradient all-reduce + clip +
  Adam kernel, captured in CUDA graphs with no host synchronisation inside ``update()``.
* **PyTorch (CPU, and model types the engine does not cover such as CNN encoders or Beta policies):** autograd,
  ``torch.optim`` and ``torch.distributed``, exactly the upstream algorithm.

Both keep parameters as ``nn.Parameter``s of the rsl_rl module layout, so ``save``/``load`` produce and accept rsl_rl
checkpoints.
"""

from __future__ import annotations

from itertools import chain

import torch
import torch.nn as nn

from ..extensions import RandomNetworkDistillation, Symmetry, resolve_rnd_config, resolve_symmetry_config
from ..models import MLPModel
from ..storage import RolloutStorage
from ..utils.utils import compile_model, reduce_gradients_in_buckets, resolve_class, resolve_obs_groups, resolve_optimizer

B200_CFG_DEFAULTS = {
    "engine": "auto",  # "auto": fused CUDA engine when supported; "torch": force the PyTorch path; "cuda": require it
    "graphs": True,  # capture act / GAE / minibatch steps in CUDA graphs
    "replica_check_interval": 0,  # >0: every k updates verify that all ranks hold bit-identical parameters
    "comm_timeout_ms": 10000,  # device-side wait limit of the peer-to-peer gradient exchange
    "exchange": "auto",  # gradient exchange: "one_shot", "two_shot", or "auto" (one shot)
    "model_streams": 2,  # 2: actor and critic kernels on two streams where independent (fork / join); 1: serial
    "rnn_fused_step": "auto",  # recurrent training steps as one launch (hidden GEMM + cell): True, False, "auto" (GRU)
    "gemm_dtype": "bf16",  # GEMM operand precision of the fused path ("bf16")
    "section_timing": False,  # time rollout / returns / update with CUDA events (Perf/section_*) and NVTX ranges
}


def resolve_b200_cfg(cfg: dict | None) -> dict:
    out = dict(B200_CFG_DEFAULTS)
    for k, v in (cfg or {}).items():
        if k not in B200_CFG_DEFAULTS:
            raise ValueError(f"Unknown b200_cfg key '{k}'. Valid keys: {list(B200_CFG_DEFAULTS)}")
        out[k] = v
    if out["rnn_fused_step"] not in (True, False, "auto"):
        raise ValueError(f"b200_cfg.rnn_fused_step must be True, False or 'auto', got {out['rnn_fused_step']!r}")
    if out["exchange"] not in ("auto", "one_shot", "two_shot"):
        raise ValueError(f"b200_cfg.exchange must be 'auto', 'one_shot' or 'two_shot', got {out['exchange']!r}")
    return out


def use_two_shot(b200_cfg: dict, world: int) -> bool:
    """Whether the fused optimizer exchanges gradients in two shots (reduce-scatter, then every rank reads each
    element's average from its owner) instead of one (every rank sums every element): fewer peer bytes per rank,
    2 (W - 1) / W instead of W - 1 vectors, for one more flag round. ``"auto"`` takes one shot: for the benchmark's
    433 k parameters the graph-replayed step measured 53.0 us one-shot and 60.8 us two-shot on 8 B200s: at this size
    the second flag round costs more than the peer bytes it saves."""
    mode = b200_cfg["exchange"]
    return world > 1 and mode == "two_shot"


# ---- the PPO objective and schedules as functions (the PyTorch path's definition; the fused kernels evaluate the same
# formulas: ops/csrc/rl_kernels.cu ppo_loss / adam_step) ------------------------------------------------------------
LR_FLOOR, LR_CEILING, LR_FACTOR = 1e-5, 1e-2, 1.5


def kl_adapted_learning_rate(lr: float, kl, desired_kl: float) -> float:
    """Adaptive-KL schedule (``rsl_rl/algorithms/ppo.py:241-266``): shrink the step when the policy moved more than
    twice the target KL, grow it when it moved less than half of it (and at all), within [1e-5, 1e-2]."""
    if kl > desired_kl * 2.0:
        return max(LR_FLOOR, lr / LR_FACTOR)
    if desired_kl / 2.0 > kl > 0.0:
        return min(LR_CEILING, lr * LR_FACTOR)
    return lr


def clipped_surrogate_loss(logp: torch.Tensor, old_logp: torch.Tensor, advantages: torch.Tensor,
                           clip: float) -> torch.Tensor:
    """Mean of ``max(-A r, -A clamp(r, 1 - clip, 1 + clip))`` with ``r = exp(logp - old_logp)``."""
    ratio = torch.exp(logp - old_logp.squeeze(-1))
    neg_adv = -advantages.squeeze(-1)
    return torch.max(neg_adv * ratio, neg_adv * torch.clamp(ratio, 1.0 - clip, 1.0 + clip)).mean()


def value_function_loss(values: torch.Tensor, old_values: torch.Tensor, returns: torch.Tensor, clip: float,
                        clipped: bool) -> torch.Tensor:
    """Squared error to the returns; with ``clipped`` the pessimistic max over the prediction and its clip to
    ``old +- clip``."""
    if not clipped:
        return (returns - values).pow(2).mean()
    near_old = old_values + (values - old_values).clamp(-clip, clip)
    return torch.max((values - returns).pow(2), (near_old - returns).pow(2)).mean()


def standardize(x: torch.Tensor) -> torch.Tensor:
    """``(x - mean) / (unbiased std + 1e-8)``."""
    return (x - x.mean()) / (x.std() + 1e-8)


def generalized_advantages(storage: RolloutStorage, last_values: torch.Tensor, gamma: float, lam: float) -> None:
    """Fill ``storage.returns`` by the reversed GAE recursion (a done cuts bootstrapping) and set
    ``storage.advantages = returns - values``."""
    values, T = storage.values, storage.num_transitions_per_env
    gae = 0
    for t in range(T - 1, -1, -1):
        bootstrap = last_values if t == T - 1 else values[t + 1]
        alive = 1.0 - storage.dones[t].float()
        delta = storage.rewards[t] + alive * gamma * bootstrap - values[t]
        gae = delta + alive * gamma * lam * gae
        storage.returns[t] = gae + values[t]
    storage.advantages = storage.returns - values


class PPO:
    """Clipped PPO with GAE, value clipping, entropy bonus, adaptive-KL learning rate and per-model gradient
    clipping; optional RND and symmetry extensions; data parallel over ranks."""

    actor: MLPModel
    critic: MLPModel

    def __init__(
        self,
        actor: MLPModel,
        critic: MLPModel,
        storage: RolloutStorage | None,
        num_learning_epochs: int = 5,
        num_mini_batches: int = 4,
        clip_param: float = 0.2,
        gamma: float = 0.99,
        lam: float = 0.95,
        value_loss_coef: float = 1.0,
        entropy_coef: float = 0.01,
        learning_rate: float = 0.001,
        max_grad_norm: float = 1.0,
        optimizer: str = "adam",
        use_clipped_value_loss: bool = True,
        schedule: str = "adaptive",
        desired_kl: float = 0.01,
        normalize_advantage_per_mini_batch: bool = False,
        use_mixed_precision: bool = False,
        device: str = "cpu",
        rnd_cfg: dict | None = None,
        symmetry_cfg: dict | None = None,
        multi_gpu_cfg: dict | None = None,
        grad_reduce_bucket_mb: float = 25,
        b200_cfg: dict | None = None,
        num_steps_per_env: int | None = None,
        num_envs: int | None = None,
        obs_template=None,
    ) -> None:
        self.device = device
        self.b200_cfg = resolve_b200_cfg(b200_cfg)
        # data parallel (one process per GPU): identity of this rank
        self.is_multi_gpu = multi_gpu_cfg is not None
        self.gpu_global_rank = multi_gpu_cfg["global_rank"] if self.is_multi_gpu else 0
        self.gpu_world_size = multi_gpu_cfg["world_size"] if self.is_multi_gpu else 1
        self.grad_reduce_bucket_mb = grad_reduce_bucket_mb
        # extensions (the RND networks draw their initial weights here, after the models')
        self.rnd = RandomNetworkDistillation(device=self.device, **rnd_cfg) if rnd_cfg else None
        if symmetry_cfg is not None and (actor.is_recurrent or critic.is_recurrent):
            raise ValueError("Symmetry augmentation is not supported for recurrent policies.")
        self.symmetry = Symmetry(**symmetry_cfg) if symmetry_cfg else None
        # models and the one optimizer over both (a shared module's parameters once)
        self.actor = self._raw_actor = actor.to(self.device)
        self.critic = self._raw_critic = critic.to(self.device)
        params = list(dict.fromkeys(chain(self.actor.parameters(), self.critic.parameters())))
        self.optimizer = resolve_optimizer(optimizer)(params, lr=learning_rate)
        self.optimizer_name = optimizer.lower()
        self.storage = storage
        self.transition = RolloutStorage.Transition()
        # hyper-parameters
        self.num_learning_epochs, self.num_mini_batches = num_learning_epochs, num_mini_batches
        self.clip_param, self.gamma, self.lam = clip_param, gamma, lam
        self.value_loss_coef, self.entropy_coef = value_loss_coef, entropy_coef
        self.max_grad_norm, self.use_clipped_value_loss = max_grad_norm, use_clipped_value_loss
        self.desired_kl, self.schedule = desired_kl, schedule
        self._learning_rate = learning_rate
        self.normalize_advantage_per_mini_batch = normalize_advantage_per_mini_batch
        self.use_mixed_precision = use_mixed_precision
        self.intrinsic_rewards: torch.Tensor | None = None
        self._obs_template = obs_template
        from ..parallel import ReplicaChecker

        self._replica_checker = ReplicaChecker(self.b200_cfg["replica_check_interval"], self.gpu_world_size)
        self.engine = None
        if self._engine_requested():
            engine_cls = _engine_class(self.actor)
            self.engine = engine_cls(self, num_steps_per_env=num_steps_per_env or storage.num_transitions_per_env,
                                     num_envs=num_envs or storage.num_envs, obs_template=obs_template)

    # ---- engine selection ---------------------------------------------------------------------------------------------
    def _engine_requested(self) -> bool:
        mode = self.b200_cfg["engine"]
        if mode == "torch" or torch.device(self.device).type != "cuda":
            if mode == "cuda":
                raise ValueError("b200_cfg.engine='cuda' requires a CUDA device")
            return False
        reason = _engine_class(self.actor).unsupported_reason(self)
        if reason is None:
            return True
        if mode == "cuda":
            raise ValueError(f"The fused CUDA engine does not support this configuration: {reason}")
        print(f"[tt_rsl_rl_b200] PPO runs on the PyTorch path: {reason}")
        return False

    # ---- learning rate (a device scalar on the fused path) ---------------------------------------------------------------
    @property
    def learning_rate(self) -> float:
        if self.engine is not None:
            return self.engine.learning_rate()
        return self._learning_rate

    @learning_rate.setter
    def learning_rate(self, value: float) -> None:
        self._learning_rate = float(value)
        if self.engine is not None:
            self.engine.set_learning_rate(float(value))

    # ---- rollout --------------------------------------------------------------------------------------------------------
    def act(self, obs) -> torch.Tensor:
        if self.engine is not None:
            return self.engine.act(obs)
        t = self.transition
        t.hidden_states = (self.actor.get_hidden_state(), self.critic.get_hidden_state())
        actions = self.actor(obs, stochastic_output=True).detach()  # draws the action noise
        t.actions = actions
        t.values = self.critic(obs).detach()
        t.actions_log_prob = self.actor.get_output_log_prob(actions).detach()
        t.distribution_params = tuple(p.detach() for p in self.actor.output_distribution_params)
        t.observations = obs
        return actions

    def process_env_step(self, obs, rewards: torch.Tensor, dones: torch.Tensor, extras: dict) -> None:
        """Store the step: reward (+ intrinsic reward, + gamma V(s) for time-outs, the bootstrap of a truncated
        episode from the value of the state it was cut in), then reset recurrent state at dones."""
        if self.engine is not None:
            self.engine.process_env_step(obs, rewards, dones, extras)
            return
        t = self.transition
        t.rewards = rewards.clone()
        t.dones = dones
        if self.rnd:
            self.intrinsic_rewards = self.rnd.get_intrinsic_reward(obs)
            t.rewards += self.intrinsic_rewards
        if "time_outs" in extras:
            truncated = extras["time_outs"].unsqueeze(1).to(self.device)
            t.rewards += self.gamma * torch.squeeze(t.values * truncated, 1)
        self.storage.add_transition(t)
        t.clear()
        self.actor.reset(dones)
        self.critic.reset(dones)

    def compute_returns(self, obs) -> None:
        if self.engine is not None:
            self.engine.compute_returns(obs)
            return
        hidden = self.critic.get_hidden_state()  # the bootstrap value must not advance the critic's state
        last_values = self.critic(obs).detach()
        self.critic.reset(hidden_state=hidden)
        st = self.storage
        generalized_advantages(st, last_values, self.gamma, self.lam)
        if not self.normalize_advantage_per_mini_batch and st.advantages.numel() > 1:
            st.advantages = standardize(st.advantages)

    # ---- update ---------------------------------------------------------------------------------------------------------
    def update(self) -> dict[str, float]:
        out = self.engine.update() if self.engine is not None else self._update_autograd()
        self._replica_checker.step(self._replicated_parameters())
        return out

    def _replicated_parameters(self):
        params = list(self.actor.parameters()) + list(self.critic.parameters())
        if self.rnd:
            params += list(self.rnd.predictor.parameters())
        return params

    def _minibatches(self):
        recurrent = self.actor.is_recurrent or self.critic.is_recurrent
        gen = self.storage.recurrent_mini_batch_generator if recurrent else self.storage.mini_batch_generator
        return gen(self.num_mini_batches, self.num_learning_epochs)

    def _update_autograd(self) -> dict[str, float]:
        keys = ["value", "surrogate", "entropy"] + (["rnd"] if self.rnd else []) + (["symmetry"] if self.symmetry
                                                                                  else [])
        totals = dict.fromkeys(keys, 0.0)
        for batch in self._minibatches():
            for key, value in self._minibatch_step(batch).items():
                totals[key] += value
        # observation statistics move only after every epoch has used the rollout's normalisation
        obs = self.storage.observations.flatten(0, 1)
        for model in (self.actor, self.critic) + ((self.rnd,) if self.rnd else ()):
            model.update_normalization(obs)
        steps = self.num_learning_epochs * self.num_mini_batches
        self.storage.clear()
        return {key: value / steps for key, value in totals.items()}

    def _adapt_learning_rate(self, batch, dist_params: tuple[torch.Tensor, ...]) -> None:
        """The adaptive-KL rule on this minibatch's mean KL (rank-averaged), before its optimizer step; rank 0
        decides and broadcasts the result."""
        with torch.inference_mode():
            kl_mean = torch.mean(self.actor.get_kl_divergence(batch.old_distribution_params, dist_params))
            if self.is_multi_gpu:
                torch.distributed.all_reduce(kl_mean, op=torch.distributed.ReduceOp.SUM)
                kl_mean /= self.gpu_world_size
            if self.gpu_global_rank == 0:
                self._learning_rate = kl_adapted_learning_rate(self._learning_rate, kl_mean, self.desired_kl)
            if self.is_multi_gpu:
                shared = torch.tensor(self._learning_rate, device=self.device)
                torch.distributed.broadcast(shared, src=0)
                self._learning_rate = shared.item()
            for group in self.optimizer.param_groups:
                group["lr"] = self._learning_rate

    def _minibatch_step(self, batch) -> dict[str, float]:
        n0 = batch.observations.batch_size[0]  # samples before symmetry copies are appended
        if self.normalize_advantage_per_mini_batch and batch.advantages.numel() > 1:
            with torch.no_grad():
                batch.advantages = standardize(batch.advantages)
        if self.symmetry:
            self.symmetry.augment_batch(batch, n0)
        device_type = torch.device(self.device).type
        with torch.amp.autocast(device_type=device_type, enabled=self.use_mixed_precision, dtype=torch.bfloat16):
            self.actor(batch.observations, masks=batch.masks, hidden_state=batch.hidden_states[0],
                       stochastic_output=True)
            logp = self.actor.get_output_log_prob(batch.actions)
            values = self.critic(batch.observations, masks=batch.masks, hidden_state=batch.hidden_states[1])
            dist_params = tuple(p[:n0] for p in self.actor.output_distribution_params)
            entropy = self.actor.output_entropy[:n0]
            if self.desired_kl is not None and self.schedule == "adaptive":
                self._adapt_learning_rate(batch, dist_params)
            surrogate = clipped_surrogate_loss(logp, batch.old_actions_log_prob, batch.advantages, self.clip_param)
            value = value_function_loss(values, batch.values, batch.returns, self.clip_param,
                                        self.use_clipped_value_loss)
            loss = surrogate + self.value_loss_coef * value - self.entropy_coef * entropy.mean()
            rnd_loss = self.rnd.compute_loss(batch.observations[:n0]) if self.rnd else None
            mirror = self.symmetry.compute_loss(self.actor, batch, n0) if self.symmetry else None
            if mirror is not None and self.symmetry.use_mirror_loss:
                loss = loss + self.symmetry.mirror_loss_coeff * mirror
        self._optimizer_step(loss, rnd_loss)
        out = {"value": value.item(), "surrogate": surrogate.item(), "entropy": entropy.mean().item()}
        if rnd_loss is not None:
            out["rnd"] = rnd_loss.item()
        if mirror is not None:
            out["symmetry"] = mirror.item()
        return out

    def _optimizer_step(self, loss: torch.Tensor, rnd_loss: torch.Tensor | None) -> None:
        """Gradients of both losses, rank average, one clip per model (actor incl. its std, critic), the steps."""
        self.optimizer.zero_grad()
        loss.backward()
        if rnd_loss is not None:
            self.rnd.optimizer.zero_grad()
            rnd_loss.backward()
        if self.is_multi_gpu:
            self.reduce_parameters()
        for model in (self.actor, self.critic):
            nn.utils.clip_grad_norm_(model.parameters(), self.max_grad_norm)
        self.optimizer.step()
        if rnd_loss is not None:
            self.rnd.optimizer.step()

    # ---- modes, checkpoints -----------------------------------------------------------------------------------------------
    def _trained_modules(self):
        return (self.actor, self.critic) + ((self.rnd,) if self.rnd else ())

    def train_mode(self) -> None:
        for m in self._trained_modules():
            m.train()

    def eval_mode(self) -> None:
        for m in self._trained_modules():
            m.eval()

    def save(self) -> dict:
        if self.engine is not None:
            self.engine.sync_to_torch()
        out = {"actor_state_dict": self._raw_actor.state_dict(), "critic_state_dict": self._raw_critic.state_dict(),
               "optimizer_state_dict": self.optimizer.state_dict()}
        if self.rnd:
            out.update(rnd_state_dict=self.rnd.state_dict(), rnd_optimizer_state_dict=self.rnd.optimizer.state_dict(),
                       rnd_update_counter=self.rnd.update_counter)
        return out

    _LOAD_ALL = {"actor": True, "critic": True, "optimizer": True, "iteration": True, "rnd": True}

    def load(self, loaded_dict: dict, load_cfg: dict | None, strict: bool) -> bool:
        """Load the selected parts (all by default); returns whether the runner resumes the iteration count."""
        if self.engine is not None:
            self.engine.sync_to_torch()
        sel = self._LOAD_ALL if load_cfg is None else load_cfg
        ckpt = _upgrade_legacy_checkpoint(loaded_dict)
        for part, model in (("actor", self._raw_actor), ("critic", self._raw_critic)):
            if sel.get(part):
                model.load_state_dict(ckpt[f"{part}_state_dict"], strict=strict)
        if sel.get("optimizer") and "optimizer_state_dict" in ckpt:
            self.optimizer.load_state_dict(ckpt["optimizer_state_dict"])
            self._learning_rate = self.optimizer.param_groups[0]["lr"]
        if sel.get("rnd") and self.rnd:
            self.rnd.load_state_dict(ckpt["rnd_state_dict"], strict=strict)
            self.rnd.optimizer.load_state_dict(ckpt["rnd_optimizer_state_dict"])
            self.rnd.update_counter = ckpt.get("rnd_update_counter", 0)
        if self.engine is not None:
            self.engine.sync_from_torch()
        return sel.get("iteration", False)

    def get_policy(self) -> MLPModel:
        if self.engine is not None:
            self.engine.sync_to_torch()
        return self._raw_actor

    def compile(self, mode: str | None = None) -> None:
        if self.engine is not None:
            if mode is not None:
                print("[tt_rsl_rl_b200] torch_compile_mode is ignored on the fused CUDA path")
            return
        self.actor = compile_model(self._raw_actor, mode)
        self.critic = compile_model(self._raw_critic, mode)

    # ---- construction ---------------------------------------------------------------------------------------------------
    @staticmethod
    def construct_algorithm(obs, env, cfg: dict, device: str) -> PPO:
        """Resolve classes and observation sets, build actor, critic, extensions and storage from a runner config."""
        alg_class, alg_cfg = resolve_class(cfg["algorithm"])
        sets = ["actor", "critic"] + (["rnd_state"] if alg_cfg.get("rnd_cfg") is not None else [])
        cfg["obs_groups"] = resolve_obs_groups(obs, cfg["obs_groups"], sets)
        alg_cfg = resolve_symmetry_config(resolve_rnd_config(alg_cfg, obs, cfg["obs_groups"], env), env)
        actor_class, actor_cfg = resolve_class(cfg["actor"])
        critic_class, critic_cfg = resolve_class(cfg["critic"])
        actor = actor_class(obs, cfg["obs_groups"], "actor", env.num_actions, **actor_cfg).to(device)
        print(f"Actor Model: {actor}")
        if alg_cfg.pop("share_cnn_encoders", None):
            critic_cfg["cnns"] = actor.cnns
        critic = critic_class(obs, cfg["obs_groups"], "critic", 1, **critic_cfg).to(device)
        print(f"Critic Model: {critic}")
        b200 = resolve_b200_cfg(alg_cfg.get("b200_cfg"))
        T = cfg["num_steps_per_env"]

        def storage():
            return RolloutStorage("rl", env.num_envs, T, obs, [env.num_actions], device)

        # the fused engine keeps its own device rollout arena: the PyTorch storage exists only when it is used
        alg = alg_class(actor, critic, None if _engine_will_run(b200, device, actor, critic, alg_cfg) else storage(),
                        device=device, **alg_cfg, multi_gpu_cfg=cfg["multi_gpu"], num_steps_per_env=T,
                        num_envs=env.num_envs, obs_template=obs)
        if alg.engine is None and alg.storage is None:
            alg.storage = storage()
        alg.compile(cfg.get("torch_compile_mode"))
        return alg

    # ---- data parallel ----------------------------------------------------------------------------------------------------
    def broadcast_parameters(self) -> None:
        """Every rank starts from rank 0's models (and RND networks)."""
        if self.engine is not None:
            self.engine.broadcast_parameters()
            return
        models = [self._raw_actor, self._raw_critic] + ([self.rnd.predictor, self.rnd.target] if self.rnd else [])
        for model in models:
            for tensor in model.state_dict().values():
                torch.distributed.broadcast(tensor, src=0)

    def reduce_parameters(self) -> None:
        """Average every trained parameter's gradient over the ranks (bucketed all-reduce)."""
        params = chain(self.actor.parameters(), self.critic.parameters())
        if self.rnd:
            params = chain(params, self.rnd.parameters())
        reduce_gradients_in_buckets(params, self.gpu_world_size, self.grad_reduce_bucket_mb)


def _engine_class(actor):
    """The fused engine for the actor's model family: recurrent (GRU/LSTM) or MLP."""
    from ..engine import PPOEngine, RecurrentPPOEngine

    return RecurrentPPOEngine if getattr(actor, "is_recurrent", False) else PPOEngine


def _engine_will_run(b200: dict, device: str, actor, critic, alg_cfg: dict) -> bool:
    if b200["engine"] == "torch" or torch.device(device).type != "cuda":
        return False
    return _engine_class(actor).supports_models(actor, critic, alg_cfg) is None


def _upgrade_legacy_checkpoint(d: dict) -> dict:
    """Accept rsl_rl <= 2.x checkpoints (``model_state_dict`` with ``actor.*``/``critic.*``/``std`` keys)."""
    if "actor_state_dict" in d or "model_state_dict" not in d:
        return d
    msd = d["model_state_dict"]
    actor_sd, critic_sd = {}, {}
    for k, v in msd.items():
        if k.startswith("actor."):
            actor_sd["mlp." + k[len("actor."):]] = v
        elif k.startswith("critic."):
            critic_sd["mlp." + k[len("critic."):]] = v
        elif k == "std":
            actor_sd["distribution.std_param"] = v
        elif k == "log_std":
            actor_sd["distribution.log_std_param"] = v
        elif k.startswith("actor_obs_normalizer."):
            actor_sd["obs_normalizer." + k.split(".", 1)[1]] = v
        elif k.startswith("critic_obs_normalizer."):
            critic_sd["obs_normalizer." + k.split(".", 1)[1]] = v
    out = dict(d)
    out["actor_state_dict"] = actor_sd
    out["critic_state_dict"] = critic_sd
    return out
