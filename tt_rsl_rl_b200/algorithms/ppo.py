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
    "gemm_dtype": "bf16",  # GEMM operand precision of the fused path ("bf16")
    "section_timing": False,  # time rollout / returns / update with CUDA events (Perf/section_*) and NVTX ranges
}


def resolve_b200_cfg(cfg: dict | None) -> dict:
    out = dict(B200_CFG_DEFAULTS)
    for k, v in (cfg or {}).items():
        if k not in B200_CFG_DEFAULTS:
            raise ValueError(f"Unknown b200_cfg key '{k}'. Valid keys: {list(B200_CFG_DEFAULTS)}")
        out[k] = v
    return out


class PPO:
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
        self.is_multi_gpu = multi_gpu_cfg is not None
        self.gpu_global_rank = multi_gpu_cfg["global_rank"] if multi_gpu_cfg else 0
        self.gpu_world_size = multi_gpu_cfg["world_size"] if multi_gpu_cfg else 1
        self.grad_reduce_bucket_mb = grad_reduce_bucket_mb
        self.b200_cfg = resolve_b200_cfg(b200_cfg)

        self.rnd = RandomNetworkDistillation(device=self.device, **rnd_cfg) if rnd_cfg else None
        if symmetry_cfg is not None and (actor.is_recurrent or critic.is_recurrent):
            raise ValueError("Symmetry augmentation is not supported for recurrent policies.")
        self.symmetry = Symmetry(**symmetry_cfg) if symmetry_cfg else None

        self.actor = actor.to(self.device)
        self.critic = critic.to(self.device)
        self._raw_actor = self.actor
        self._raw_critic = self.critic
        self.optimizer = resolve_optimizer(optimizer)(
            list(dict.fromkeys(chain(self.actor.parameters(), self.critic.parameters()))), lr=learning_rate
        )
        self.optimizer_name = optimizer.lower()
        self.storage = storage
        self.transition = RolloutStorage.Transition()

        self.clip_param = clip_param
        self.num_learning_epochs = num_learning_epochs
        self.num_mini_batches = num_mini_batches
        self.value_loss_coef = value_loss_coef
        self.entropy_coef = entropy_coef
        self.gamma = gamma
        self.lam = lam
        self.max_grad_norm = max_grad_norm
        self.use_clipped_value_loss = use_clipped_value_loss
        self.desired_kl = desired_kl
        self.schedule = schedule
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
        self.transition.hidden_states = (self.actor.get_hidden_state(), self.critic.get_hidden_state())
        self.transition.actions = self.actor(obs, stochastic_output=True).detach()
        self.transition.values = self.critic(obs).detach()
        self.transition.actions_log_prob = self.actor.get_output_log_prob(self.transition.actions).detach()
        self.transition.distribution_params = tuple(p.detach() for p in self.actor.output_distribution_params)
        self.transition.observations = obs
        return self.transition.actions

    def process_env_step(self, obs, rewards: torch.Tensor, dones: torch.Tensor, extras: dict) -> None:
        if self.engine is not None:
            self.engine.process_env_step(obs, rewards, dones, extras)
            return
        self.transition.rewards = rewards.clone()
        self.transition.dones = dones
        if self.rnd:
            self.intrinsic_rewards = self.rnd.get_intrinsic_reward(obs)
            self.transition.rewards += self.intrinsic_rewards
        if "time_outs" in extras:
            # bootstrap truncated episodes with the value of the state they were cut in
            self.transition.rewards += self.gamma * torch.squeeze(
                self.transition.values * extras["time_outs"].unsqueeze(1).to(self.device), 1
            )
        self.storage.add_transition(self.transition)
        self.transition.clear()
        self.actor.reset(dones)
        self.critic.reset(dones)

    def compute_returns(self, obs) -> None:
        if self.engine is not None:
            self.engine.compute_returns(obs)
            return
        st = self.storage
        hidden = self.critic.get_hidden_state()
        last_values = self.critic(obs).detach()
        self.critic.reset(hidden_state=hidden)
        gae = 0
        T = st.num_transitions_per_env
        for t in reversed(range(T)):
            next_values = last_values if t == T - 1 else st.values[t + 1]
            not_done = 1.0 - st.dones[t].float()
            delta = st.rewards[t] + not_done * self.gamma * next_values - st.values[t]
            gae = delta + not_done * self.gamma * self.lam * gae
            st.returns[t] = gae + st.values[t]
        st.advantages = st.returns - st.values
        if not self.normalize_advantage_per_mini_batch and st.advantages.numel() > 1:
            st.advantages = (st.advantages - st.advantages.mean()) / (st.advantages.std() + 1e-8)

    # ---- update ---------------------------------------------------------------------------------------------------------
    def update(self) -> dict[str, float]:
        out = self._update()
        self._replica_checker.step(self._replicated_parameters())
        return out

    def _replicated_parameters(self):
        params = list(self.actor.parameters()) + list(self.critic.parameters())
        if self.rnd:
            params += list(self.rnd.predictor.parameters())
        return params

    def _update(self) -> dict[str, float]:
        if self.engine is not None:
            return self.engine.update()
        sums = {"value": 0.0, "surrogate": 0.0, "entropy": 0.0}
        if self.rnd:
            sums["rnd"] = 0.0
        if self.symmetry:
            sums["symmetry"] = 0.0
        if self.actor.is_recurrent or self.critic.is_recurrent:
            batches = self.storage.recurrent_mini_batch_generator(self.num_mini_batches, self.num_learning_epochs)
        else:
            batches = self.storage.mini_batch_generator(self.num_mini_batches, self.num_learning_epochs)
        for batch in batches:
            terms = self._minibatch_step(batch)
            for k, v in terms.items():
                sums[k] += v
        obs = self.storage.observations.flatten(0, 1)
        self.actor.update_normalization(obs)
        self.critic.update_normalization(obs)
        if self.rnd:
            self.rnd.update_normalization(obs)
        n = self.num_learning_epochs * self.num_mini_batches
        self.storage.clear()
        return {k: v / n for k, v in sums.items()}

    def _adapt_learning_rate(self, batch, dist_params: tuple[torch.Tensor, ...]) -> None:
        """Adaptive-KL schedule, evaluated every minibatch before its optimizer step (``ppo.py:241-266``)."""
        with torch.inference_mode():
            kl_mean = torch.mean(self.actor.get_kl_divergence(batch.old_distribution_params, dist_params))
            if self.is_multi_gpu:
                torch.distributed.all_reduce(kl_mean, op=torch.distributed.ReduceOp.SUM)
                kl_mean /= self.gpu_world_size
            if self.gpu_global_rank == 0:
                if kl_mean > self.desired_kl * 2.0:
                    self._learning_rate = max(1e-5, self._learning_rate / 1.5)
                elif self.desired_kl / 2.0 > kl_mean > 0.0:
                    self._learning_rate = min(1e-2, self._learning_rate * 1.5)
            if self.is_multi_gpu:
                lr = torch.tensor(self._learning_rate, device=self.device)
                torch.distributed.broadcast(lr, src=0)
                self._learning_rate = lr.item()
            for group in self.optimizer.param_groups:
                group["lr"] = self._learning_rate

    def _minibatch_step(self, batch) -> dict[str, float]:
        n0 = batch.observations.batch_size[0]
        if self.normalize_advantage_per_mini_batch and batch.advantages.numel() > 1:
            with torch.no_grad():
                batch.advantages = (batch.advantages - batch.advantages.mean()) / (batch.advantages.std() + 1e-8)
        if self.symmetry:
            self.symmetry.augment_batch(batch, n0)
        with torch.amp.autocast(device_type=torch.device(self.device).type, enabled=self.use_mixed_precision,
                                dtype=torch.bfloat16):
            self.actor(batch.observations, masks=batch.masks, hidden_state=batch.hidden_states[0],
                       stochastic_output=True)
            logp = self.actor.get_output_log_prob(batch.actions)
            values = self.critic(batch.observations, masks=batch.masks, hidden_state=batch.hidden_states[1])
            dist_params = tuple(p[:n0] for p in self.actor.output_distribution_params)
            entropy = self.actor.output_entropy[:n0]
            if self.desired_kl is not None and self.schedule == "adaptive":
                self._adapt_learning_rate(batch, dist_params)
            ratio = torch.exp(logp - batch.old_actions_log_prob.squeeze(-1))
            adv = batch.advantages.squeeze(-1)
            surrogate_loss = torch.max(-adv * ratio,
                                       -adv * torch.clamp(ratio, 1.0 - self.clip_param, 1.0 + self.clip_param)).mean()
            if self.use_clipped_value_loss:
                clipped = batch.values + (values - batch.values).clamp(-self.clip_param, self.clip_param)
                value_loss = torch.max((values - batch.returns).pow(2), (clipped - batch.returns).pow(2)).mean()
            else:
                value_loss = (batch.returns - values).pow(2).mean()
            loss = surrogate_loss + self.value_loss_coef * value_loss - self.entropy_coef * entropy.mean()
            rnd_loss = self.rnd.compute_loss(batch.observations[:n0]) if self.rnd else None
            symmetry_loss = None
            if self.symmetry:
                symmetry_loss = self.symmetry.compute_loss(self.actor, batch, n0)
                if self.symmetry.use_mirror_loss:
                    loss = loss + self.symmetry.mirror_loss_coeff * symmetry_loss
        self.optimizer.zero_grad()
        loss.backward()
        if self.rnd:
            self.rnd.optimizer.zero_grad()
            rnd_loss.backward()
        if self.is_multi_gpu:
            self.reduce_parameters()
        nn.utils.clip_grad_norm_(self.actor.parameters(), self.max_grad_norm)
        nn.utils.clip_grad_norm_(self.critic.parameters(), self.max_grad_norm)
        self.optimizer.step()
        if self.rnd:
            self.rnd.optimizer.step()
        out = {"value": value_loss.item(), "surrogate": surrogate_loss.item(), "entropy": entropy.mean().item()}
        if rnd_loss is not None:
            out["rnd"] = rnd_loss.item()
        if symmetry_loss is not None:
            out["symmetry"] = symmetry_loss.item()
        return out

    # ---- modes, checkpoints -----------------------------------------------------------------------------------------------
    def train_mode(self) -> None:
        self.actor.train()
        self.critic.train()
        if self.rnd:
            self.rnd.train()

    def eval_mode(self) -> None:
        self.actor.eval()
        self.critic.eval()
        if self.rnd:
            self.rnd.eval()

    def save(self) -> dict:
        if self.engine is not None:
            self.engine.sync_to_torch()
        out = {
            "actor_state_dict": self._raw_actor.state_dict(),
            "critic_state_dict": self._raw_critic.state_dict(),
            "optimizer_state_dict": self.optimizer.state_dict(),
        }
        if self.rnd:
            out["rnd_state_dict"] = self.rnd.state_dict()
            out["rnd_optimizer_state_dict"] = self.rnd.optimizer.state_dict()
            out["rnd_update_counter"] = self.rnd.update_counter
        return out

    def load(self, loaded_dict: dict, load_cfg: dict | None, strict: bool) -> bool:
        if self.engine is not None:
            self.engine.sync_to_torch()
        if load_cfg is None:
            load_cfg = {"actor": True, "critic": True, "optimizer": True, "iteration": True, "rnd": True}
        loaded_dict = _upgrade_legacy_checkpoint(loaded_dict)
        if load_cfg.get("actor"):
            self._raw_actor.load_state_dict(loaded_dict["actor_state_dict"], strict=strict)
        if load_cfg.get("critic"):
            self._raw_critic.load_state_dict(loaded_dict["critic_state_dict"], strict=strict)
        if load_cfg.get("optimizer") and "optimizer_state_dict" in loaded_dict:
            self.optimizer.load_state_dict(loaded_dict["optimizer_state_dict"])
            self._learning_rate = self.optimizer.param_groups[0]["lr"]
        if load_cfg.get("rnd") and self.rnd:
            self.rnd.load_state_dict(loaded_dict["rnd_state_dict"], strict=strict)
            self.rnd.optimizer.load_state_dict(loaded_dict["rnd_optimizer_state_dict"])
            self.rnd.update_counter = loaded_dict.get("rnd_update_counter", 0)
        if self.engine is not None:
            self.engine.sync_from_torch()
        return load_cfg.get("iteration", False)

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
        alg_class, alg_cfg = resolve_class(cfg["algorithm"])
        actor_class, actor_cfg = resolve_class(cfg["actor"])
        critic_class, critic_cfg = resolve_class(cfg["critic"])
        default_sets = ["actor", "critic"]
        if alg_cfg.get("rnd_cfg") is not None:
            default_sets.append("rnd_state")
        cfg["obs_groups"] = resolve_obs_groups(obs, cfg["obs_groups"], default_sets)
        alg_cfg = resolve_rnd_config(alg_cfg, obs, cfg["obs_groups"], env)
        alg_cfg = resolve_symmetry_config(alg_cfg, env)
        actor = actor_class(obs, cfg["obs_groups"], "actor", env.num_actions, **actor_cfg).to(device)
        print(f"Actor Model: {actor}")
        if alg_cfg.pop("share_cnn_encoders", None):
            critic_cfg["cnns"] = actor.cnns
        critic = critic_class(obs, cfg["obs_groups"], "critic", 1, **critic_cfg).to(device)
        print(f"Critic Model: {critic}")
        b200 = resolve_b200_cfg(alg_cfg.get("b200_cfg"))
        # The fused engine keeps its own device rollout arena; the PyTorch storage is only allocated when needed.
        storage = None
        if not _engine_will_run(b200, device, actor, critic, alg_cfg):
            storage = RolloutStorage("rl", env.num_envs, cfg["num_steps_per_env"], obs, [env.num_actions], device)
        alg = alg_class(actor, critic, storage, device=device, **alg_cfg, multi_gpu_cfg=cfg["multi_gpu"],
                        num_steps_per_env=cfg["num_steps_per_env"], num_envs=env.num_envs, obs_template=obs)
        if alg.engine is None and alg.storage is None:
            alg.storage = RolloutStorage("rl", env.num_envs, cfg["num_steps_per_env"], obs, [env.num_actions], device)
        alg.compile(cfg.get("torch_compile_mode"))
        return alg

    # ---- data parallel ----------------------------------------------------------------------------------------------------
    def broadcast_parameters(self) -> None:
        if self.engine is not None:
            self.engine.broadcast_parameters()
            return
        models = [self._raw_actor, self._raw_critic]
        if self.rnd:
            models += [self.rnd.predictor, self.rnd.target]
        for model in models:
            for tensor in model.state_dict().values():
                torch.distributed.broadcast(tensor, src=0)

    def reduce_parameters(self) -> None:
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
