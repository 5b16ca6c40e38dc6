"""Distillation runner (``rsl_rl/runners/distillation_runner.py``): refuses to learn before a teacher is loaded."""

from __future__ import annotations

from ..algorithms import Distillation
from .on_policy_runner import OnPolicyRunner


class DistillationRunner(OnPolicyRunner):
    alg: Distillation

    def learn(self, num_learning_iterations: int, init_at_random_ep_len: bool = False) -> None:
        if not self.alg.teacher_loaded:
            raise ValueError("Teacher model parameters not loaded. Please load a teacher model to distill.")
        super().learn(num_learning_iterations, init_at_random_ep_len)
