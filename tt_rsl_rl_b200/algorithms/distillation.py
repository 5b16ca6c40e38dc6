"""Student-teacher distillation by behaviour cloning.

Interface: rsl_rl's ``Distillation`` (``rsl_rl/algorithms/distillation.py``) -- constructor arguments, the algorithm
protocol the runner drives (``act`` / ``process_env_step`` / ``compute_returns`` / ``update`` / ``save`` / ``load`` /
``broadcast_parameters`` / ...), the checkpoint keys ``student_state_dict``, ``teacher_state_dict`` and
``optimizer_state_dict``, and teacher loading from an RL checkpoint (its ``actor_state_dict``).

Training signal (the window rule, ``distillation.py:143-201``): the storage yields one batch per rollout step; the
behaviour-cloning losses of ``gradient_length`` consecutive steps are *summed* and applied as one optimizer step, so a
window's gradient is the sum of its steps' gradients; steps that do not fill a last window are dropped. A recurrent
student carries its hidden state through the rollout, resets it at dones, and is detached at every window boundary
(truncated backpropagation through time).

Execution: on CUDA :class:`tt_rsl_rl_b200.engine.DistillationEngine` (MLP student) or
:class:`tt_rsl_rl_b200.engine.RecurrentDistillationEngine` (GRU / LSTM student), with an MLP or recurrent teacher,
runs the step in the framework's kernels (forward / backward GEMMs with persistent fp32 gradient sums, fused clip +
Adam); otherwise :class:`_LossWindow` below drives autograd.
"""

from __future__ import annotations

import warnings
from typing import Callable

import torch
import torch.nn as nn

from ..models import MLPModel
from ..storage import RolloutStorage
from ..utils.utils import compile_model, reduce_gradients_in_buckets, resolve_class, resolve_obs_groups, resolve_optimizer
from .ppo import resolve_b200_cfg

_LOSSES: dict[str, Callable] = {"mse": nn.functional.mse_loss, "huber": nn.functional.huber_loss}


class _LossWindow:
    """Sums step losses and hands every ``length``-th running sum to ``apply`` (one optimizer step)."""

    def __init__(self, length: int, apply: Callable[[torch.Tensor], None]) -> None:
        self.length = length
        self.apply = apply
        self.steps = 0
        self.total: torch.Tensor | None = None
        self.values: list[float] = []  # every step's loss value, for logging

    def add(self, loss: torch.Tensor) -> None:
        self.total = loss if self.total is None else self.total + loss
        self.values.append(loss.item())
        self.steps += 1
        if self.steps % self.length == 0:
            self.apply(self.total)
            self.total = None

    def mean(self) -> float:
        return sum(self.values) / len(self.values)


class Distillation:
    student: MLPModel
    teacher: MLPModel
    teacher_loaded: bool = False

    def __init__(
        self,
        student: MLPModel,
        teacher: MLPModel,
        storage: RolloutStorage,
        num_learning_epochs: int = 1,
        gradient_length: int = 15,
        learning_rate: float = 1e-3,
        max_grad_norm: float | None = None,
        loss_type: str = "mse",
        optimizer: str = "adam",
        use_mixed_precision: bool = False,
        device: str = "cpu",
        multi_gpu_cfg: dict | None = None,
        grad_reduce_bucket_mb: float = 25,
        b200_cfg: dict | None = None,
        **kwargs,
    ) -> None:
        if loss_type not in _LOSSES:
            raise ValueError(f"loss_type {loss_type!r} is not one of {sorted(_LOSSES)}")
        self.device = device
        self.b200_cfg = resolve_b200_cfg(b200_cfg)
        # data parallel (one process per GPU): identity of this rank
        self.is_multi_gpu = multi_gpu_cfg is not None
        self.gpu_global_rank = multi_gpu_cfg["global_rank"] if self.is_multi_gpu else 0
        self.gpu_world_size = multi_gpu_cfg["world_size"] if self.is_multi_gpu else 1
        self.grad_reduce_bucket_mb = grad_reduce_bucket_mb
        # models (the raw modules stay reachable when ``compile`` wraps them)
        self.student = self._raw_student = student.to(device)
        self.teacher = self._raw_teacher = teacher.to(device)
        self.optimizer_name = optimizer
        self.optimizer = resolve_optimizer(optimizer)(self.student.parameters(), lr=learning_rate)
        self.storage = storage
        self.transition = RolloutStorage.Transition()
        self.last_student_hidden_state = None
        # hyper-parameters
        self.num_learning_epochs = num_learning_epochs
        self.gradient_length = gradient_length
        self.learning_rate = learning_rate
        self.max_grad_norm = max_grad_norm
        self.use_mixed_precision = use_mixed_precision
        self.loss_type = loss_type
        self.loss_fn = _LOSSES[loss_type]
        self.num_updates = 0
        self._warn_about_dropped_steps(num_learning_epochs * storage.num_transitions_per_env)
        from ..parallel import ReplicaChecker

        self._replica_checker = ReplicaChecker(self.b200_cfg["replica_check_interval"], self.gpu_world_size)
        self.engine = self._select_engine()

    def _warn_about_dropped_steps(self, steps: int) -> None:
        dropped = steps % self.gradient_length
        if dropped:
            warnings.warn(
                f"gradient_length={self.gradient_length} does not divide the {steps} behaviour-cloning steps of an "
                f"update (num_learning_epochs x num_steps_per_env): the losses of the last {dropped} steps are "
                f"summed but never applied. A divisor of {steps} uses every step.",
                stacklevel=3,
            )

    def _select_engine(self):
        mode = self.b200_cfg["engine"]
        if mode == "torch" or torch.device(self.device).type != "cuda":
            return None
        from ..engine.distillation_engine import DistillationEngine, RecurrentDistillationEngine
        from ..models import RNNModel

        cls = RecurrentDistillationEngine if isinstance(self.student, RNNModel) else DistillationEngine
        reason = cls.unsupported_reason(self)
        if reason is None:
            return cls(self)
        if mode == "cuda":
            raise ValueError(f"The fused CUDA distillation engine does not support this configuration: {reason}")
        return None

    # ---- rollout ------------------------------------------------------------------------------------------------------
    def act(self, obs) -> torch.Tensor:
        if self.engine is not None:
            return self.engine.act(obs)
        t = self.transition
        t.actions = self.student(obs, stochastic_output=True).detach()
        t.privileged_actions = self.teacher(obs).detach()
        t.observations = obs
        return t.actions

    def process_env_step(self, obs, rewards: torch.Tensor, dones: torch.Tensor, extras: dict) -> None:
        if self.engine is not None:
            self.engine.process_env_step(obs, rewards, dones, extras)
            return
        self.transition.rewards, self.transition.dones = rewards, dones
        self.storage.add_transition(self.transition)
        self.transition.clear()
        for model in (self.student, self.teacher):
            model.reset(dones)

    def compute_returns(self, obs) -> None:
        """Behaviour cloning has no return targets."""

    # ---- update -------------------------------------------------------------------------------------------------------
    def update(self) -> dict[str, float]:
        self.num_updates += 1
        if self.engine is not None:
            losses = self.engine.update()
            self.storage.clear()
        else:
            losses = {"behavior": self._update_autograd()}
        self._replica_checker.step(list(self.student.parameters()))
        return losses

    def _behaviour_loss(self, batch) -> torch.Tensor:
        device_type = torch.device(self.device).type
        with torch.amp.autocast(device_type=device_type, enabled=self.use_mixed_precision, dtype=torch.bfloat16):
            return self.loss_fn(self.student(batch.observations), batch.privileged_actions)

    def _apply_window(self, window_loss: torch.Tensor) -> None:
        """One optimizer step on a window's summed loss (rank-averaged gradients, optional clip)."""
        self.optimizer.zero_grad()
        window_loss.backward()
        if self.is_multi_gpu:
            self.reduce_parameters()
        if self.max_grad_norm:
            nn.utils.clip_grad_norm_(self.student.parameters(), self.max_grad_norm)
        self.optimizer.step()
        self.student.detach_hidden_state()  # truncate backpropagation at the window boundary

    def _update_autograd(self) -> float:
        window = _LossWindow(self.gradient_length, self._apply_window)
        student = self.student
        for _ in range(self.num_learning_epochs):
            # every epoch replays the rollout from the hidden state the student had when it started
            student.reset(hidden_state=self.last_student_hidden_state)
            student.detach_hidden_state()
            for batch in self.storage.generator():
                window.add(self._behaviour_loss(batch))
                done = batch.dones.view(-1)
                student.reset(done)
                student.detach_hidden_state(done)
        self.last_student_hidden_state = student.get_hidden_state()
        student.detach_hidden_state()
        student.update_normalization(self.storage.observations.flatten(0, 1))
        self.storage.clear()
        return window.mean()

    # ---- modes, checkpoints ---------------------------------------------------------------------------------------
    def train_mode(self) -> None:
        self.student.train()
        self.teacher.eval()  # the teacher is never trained

    def eval_mode(self) -> None:
        self.student.eval()
        self.teacher.eval()

    def save(self) -> dict:
        if self.engine is not None:
            self.engine.sync_to_torch()
        return {"student_state_dict": self._raw_student.state_dict(),
                "teacher_state_dict": self._raw_teacher.state_dict(),
                "optimizer_state_dict": self.optimizer.state_dict()}

    @staticmethod
    def _default_load_cfg(loaded: dict) -> dict:
        """An RL checkpoint (it has an actor) provides only the teacher; a distillation checkpoint provides all."""
        if any("actor_state_dict" in key for key in loaded):
            return {"teacher": True, "iteration": False}
        return {"student": True, "teacher": True, "optimizer": True, "iteration": True}

    def load(self, loaded_dict: dict, load_cfg: dict | None, strict: bool) -> bool:
        """Load the selected parts; returns whether the runner should resume the checkpoint's iteration count."""
        if self.engine is not None:
            self.engine.sync_to_torch()
        sel = self._default_load_cfg(loaded_dict) if load_cfg is None else load_cfg
        if sel.get("student"):
            self._raw_student.load_state_dict(loaded_dict["student_state_dict"], strict=strict)
        if sel.get("teacher"):
            teacher_sd = loaded_dict.get("teacher_state_dict") or loaded_dict["actor_state_dict"]
            self._raw_teacher.load_state_dict(teacher_sd, strict=strict)
            self.teacher_loaded = True
        if sel.get("optimizer"):
            self.optimizer.load_state_dict(loaded_dict["optimizer_state_dict"])
        if self.engine is not None:
            self.engine.sync_from_torch()
        return sel.get("iteration", False)

    def get_policy(self) -> MLPModel:
        return self._raw_student

    def compile(self, mode: str | None = None) -> None:
        self.student = compile_model(self._raw_student, mode)
        self.teacher = compile_model(self._raw_teacher, mode)

    # ---- construction from a runner configuration -------------------------------------------------------------------
    @staticmethod
    def construct_algorithm(obs, env, cfg: dict, device: str) -> Distillation:
        alg_class, alg_cfg = resolve_class(cfg["algorithm"])
        cfg["obs_groups"] = resolve_obs_groups(obs, cfg["obs_groups"], ["student", "teacher"])
        for ext in ("rnd_cfg", "symmetry_cfg"):
            if alg_cfg.get(ext) is not None:
                name = "RND" if ext == "rnd_cfg" else "symmetry"
                raise ValueError(f"The {name} extension is not compatible with Distillation.")
            alg_cfg[ext] = None
        models = {}
        for role in ("student", "teacher"):
            model_class, model_cfg = resolve_class(cfg[role])
            models[role] = model_class(obs, cfg["obs_groups"], role, env.num_actions, **model_cfg).to(device)
            print(f"{role.capitalize()} Model: {models[role]}")
        storage = RolloutStorage("distillation", env.num_envs, cfg["num_steps_per_env"], obs, [env.num_actions],
                                 device)
        alg = alg_class(models["student"], models["teacher"], storage, device=device, **alg_cfg,
                        multi_gpu_cfg=cfg["multi_gpu"])
        alg.compile(cfg.get("torch_compile_mode"))
        return alg

    # ---- data parallel -------------------------------------------------------------------------------------------------
    def broadcast_parameters(self) -> None:
        """Every rank starts from rank 0's student and teacher."""
        if self.engine is not None:
            self.engine.broadcast_parameters()
            return
        for model in (self._raw_student, self._raw_teacher):
            for tensor in model.state_dict().values():
                torch.distributed.broadcast(tensor, src=0)

    def reduce_parameters(self) -> None:
        """Average the student's gradients over the ranks."""
        reduce_gradients_in_buckets(self.student.parameters(), self.gpu_world_size, self.grad_reduce_bucket_mb)
