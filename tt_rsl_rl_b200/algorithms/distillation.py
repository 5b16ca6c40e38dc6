"""Student-teacher distillation by behaviour cloning (``rsl_rl/algorithms/distillation.py``).

Gradients of a window are the *sum* of the per-step losses' gradients over ``gradient_length`` consecutive steps;
leftover steps at the end of an update are accumulated but never applied (``distillation.py:93-102``).
On CUDA with MLP student/teacher, :class:`tt_rsl_rl_b200.engine.DistillationEngine` runs the step with the framework's
kernels (forward/backward GEMMs with persistent fp32 gradient accumulation, fused clip + Adam).
"""

from __future__ import annotations

import warnings

import torch
import torch.nn as nn

from ..models import MLPModel
from ..storage import RolloutStorage
from ..utils.utils import compile_model, reduce_gradients_in_buckets, resolve_class, resolve_obs_groups, resolve_optimizer
from .ppo import resolve_b200_cfg


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
        self.device = device
        self.is_multi_gpu = multi_gpu_cfg is not None
        self.gpu_global_rank = multi_gpu_cfg["global_rank"] if multi_gpu_cfg else 0
        self.gpu_world_size = multi_gpu_cfg["world_size"] if multi_gpu_cfg else 1
        self.grad_reduce_bucket_mb = grad_reduce_bucket_mb
        self.b200_cfg = resolve_b200_cfg(b200_cfg)
        self.student = student.to(device)
        self.teacher = teacher.to(device)
        self._raw_student = self.student
        self._raw_teacher = self.teacher
        self.optimizer_name = optimizer
        self.optimizer = resolve_optimizer(optimizer)(self.student.parameters(), lr=learning_rate)
        self.storage = storage
        self.transition = RolloutStorage.Transition()
        self.last_student_hidden_state = None
        self.num_learning_epochs = num_learning_epochs
        self.gradient_length = gradient_length
        self.learning_rate = learning_rate
        self.max_grad_norm = max_grad_norm
        self.use_mixed_precision = use_mixed_precision
        self.loss_type = loss_type
        total = num_learning_epochs * storage.num_transitions_per_env
        if total % gradient_length != 0:
            warnings.warn(
                f"The product of 'num_learning_epochs' ({num_learning_epochs}) and 'num_steps_per_env'"
                f" ({storage.num_transitions_per_env}) is not divisible by 'gradient_length' ({gradient_length})."
                f" The last {total % gradient_length} of {total} steps per update are accumulated but never"
                f" backpropagated. Consider setting 'gradient_length' to a divisor of {total}.",
                stacklevel=2,
            )
        losses = {"mse": nn.functional.mse_loss, "huber": nn.functional.huber_loss}
        if loss_type not in losses:
            raise ValueError(f"Unknown loss type: {loss_type}. Supported types are: {list(losses)}")
        self.loss_fn = losses[loss_type]
        self.num_updates = 0
        from ..parallel import ReplicaChecker

        self._replica_checker = ReplicaChecker(self.b200_cfg["replica_check_interval"], self.gpu_world_size)
        self.engine = None
        if self.b200_cfg["engine"] != "torch" and torch.device(device).type == "cuda":
            from ..engine.distillation_engine import DistillationEngine

            reason = DistillationEngine.unsupported_reason(self)
            if reason is None:
                self.engine = DistillationEngine(self)
            elif self.b200_cfg["engine"] == "cuda":
                raise ValueError(f"The fused CUDA distillation engine does not support this configuration: {reason}")

    def act(self, obs) -> torch.Tensor:
        if self.engine is not None:
            return self.engine.act(obs)
        self.transition.actions = self.student(obs, stochastic_output=True).detach()
        self.transition.privileged_actions = self.teacher(obs).detach()
        self.transition.observations = obs
        return self.transition.actions

    def process_env_step(self, obs, rewards: torch.Tensor, dones: torch.Tensor, extras: dict) -> None:
        if self.engine is not None:
            self.engine.process_env_step(obs, rewards, dones, extras)
            return
        self.transition.rewards = rewards
        self.transition.dones = dones
        self.storage.add_transition(self.transition)
        self.transition.clear()
        self.student.reset(dones)
        self.teacher.reset(dones)

    def compute_returns(self, obs) -> None:
        """Distillation needs no return targets."""

    def update(self) -> dict[str, float]:
        out = self._update()
        self._replica_checker.step(list(self.student.parameters()))
        return out

    def _update(self) -> dict[str, float]:
        self.num_updates += 1
        if self.engine is not None:
            loss_dict = self.engine.update()
            self.storage.clear()
            return loss_dict
        total_loss = 0.0
        window_loss = 0
        count = 0
        for _ in range(self.num_learning_epochs):
            self.student.reset(hidden_state=self.last_student_hidden_state)
            self.student.detach_hidden_state()
            for batch in self.storage.generator():
                with torch.amp.autocast(device_type=torch.device(self.device).type,
                                        enabled=self.use_mixed_precision, dtype=torch.bfloat16):
                    actions = self.student(batch.observations)
                    step_loss = self.loss_fn(actions, batch.privileged_actions)
                window_loss = window_loss + step_loss
                total_loss += step_loss.item()
                count += 1
                if count % self.gradient_length == 0:
                    self.optimizer.zero_grad()
                    window_loss.backward()
                    if self.is_multi_gpu:
                        self.reduce_parameters()
                    if self.max_grad_norm:
                        nn.utils.clip_grad_norm_(self.student.parameters(), self.max_grad_norm)
                    self.optimizer.step()
                    self.student.detach_hidden_state()
                    window_loss = 0
                self.student.reset(batch.dones.view(-1))
                self.student.detach_hidden_state(batch.dones.view(-1))
        self.last_student_hidden_state = self.student.get_hidden_state()
        self.student.detach_hidden_state()
        self.student.update_normalization(self.storage.observations.flatten(0, 1))
        self.storage.clear()
        return {"behavior": total_loss / count}

    def train_mode(self) -> None:
        self.student.train()
        self.teacher.eval()

    def eval_mode(self) -> None:
        self.student.eval()
        self.teacher.eval()

    def save(self) -> dict:
        if self.engine is not None:
            self.engine.sync_to_torch()
        return {
            "student_state_dict": self._raw_student.state_dict(),
            "teacher_state_dict": self._raw_teacher.state_dict(),
            "optimizer_state_dict": self.optimizer.state_dict(),
        }

    def load(self, loaded_dict: dict, load_cfg: dict | None, strict: bool) -> bool:
        if self.engine is not None:
            self.engine.sync_to_torch()
        resume = self._load(loaded_dict, load_cfg, strict)
        if self.engine is not None:
            self.engine.sync_from_torch()
        return resume

    def _load(self, loaded_dict: dict, load_cfg: dict | None, strict: bool) -> bool:
        if load_cfg is None:
            if any("actor_state_dict" in k for k in loaded_dict):
                load_cfg = {"teacher": True, "iteration": False}
            else:
                load_cfg = {"student": True, "teacher": True, "optimizer": True, "iteration": True}
        if load_cfg.get("student"):
            self._raw_student.load_state_dict(loaded_dict["student_state_dict"], strict=strict)
        if load_cfg.get("teacher"):
            sd = loaded_dict.get("teacher_state_dict") or loaded_dict["actor_state_dict"]
            self._raw_teacher.load_state_dict(sd, strict=strict)
            self.teacher_loaded = True
        if load_cfg.get("optimizer"):
            self.optimizer.load_state_dict(loaded_dict["optimizer_state_dict"])
        return load_cfg.get("iteration", False)

    def get_policy(self) -> MLPModel:
        return self._raw_student

    def compile(self, mode: str | None = None) -> None:
        self.student = compile_model(self._raw_student, mode)
        self.teacher = compile_model(self._raw_teacher, mode)

    @staticmethod
    def construct_algorithm(obs, env, cfg: dict, device: str) -> Distillation:
        alg_class, alg_cfg = resolve_class(cfg["algorithm"])
        student_class, student_cfg = resolve_class(cfg["student"])
        teacher_class, teacher_cfg = resolve_class(cfg["teacher"])
        cfg["obs_groups"] = resolve_obs_groups(obs, cfg["obs_groups"], ["student", "teacher"])
        if alg_cfg.get("rnd_cfg") is not None:
            raise ValueError("The RND extension is not compatible with Distillation.")
        alg_cfg["rnd_cfg"] = None
        if alg_cfg.get("symmetry_cfg") is not None:
            raise ValueError("The symmetry extension is not compatible with Distillation.")
        alg_cfg["symmetry_cfg"] = None
        student = student_class(obs, cfg["obs_groups"], "student", env.num_actions, **student_cfg).to(device)
        print(f"Student Model: {student}")
        teacher = teacher_class(obs, cfg["obs_groups"], "teacher", env.num_actions, **teacher_cfg).to(device)
        print(f"Teacher Model: {teacher}")
        storage = RolloutStorage("distillation", env.num_envs, cfg["num_steps_per_env"], obs, [env.num_actions],
                                 device)
        alg = alg_class(student, teacher, storage, device=device, **alg_cfg, multi_gpu_cfg=cfg["multi_gpu"])
        alg.compile(cfg.get("torch_compile_mode"))
        return alg

    def broadcast_parameters(self) -> None:
        if self.engine is not None:
            self.engine.broadcast_parameters()
            return
        for model in (self._raw_student, self._raw_teacher):
            for tensor in model.state_dict().values():
                torch.distributed.broadcast(tensor, src=0)

    def reduce_parameters(self) -> None:
        reduce_gradients_in_buckets(self.student.parameters(), self.gpu_world_size, self.grad_reduce_bucket_mb)
