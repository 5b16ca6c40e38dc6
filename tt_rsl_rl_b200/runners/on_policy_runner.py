"""On-policy runner (``rsl_rl/runners/on_policy_runner.py``): rollout / update loop, checkpoints, export, multi-GPU.

Multi-GPU runs one process per GPU launched by ``torchrun`` (``WORLD_SIZE``, ``RANK``, ``LOCAL_RANK``), as upstream.
``torch.distributed`` (NCCL on CUDA, gloo on CPU) is the bootstrap; on the fused CUDA path the gradient exchange,
parameter broadcast and normaliser statistics go through the framework's peer-to-peer communicator instead
(``tt_rsl_rl_b200/parallel``).

With the fused engine and an environment that declares ``graph_capturable``, a whole rollout (``T`` x (act, env step,
store, episode bookkeeping)) is captured once and replayed as a single CUDA graph per iteration.
"""

from __future__ import annotations

import os
import re
import time

import torch

from ..algorithms import PPO
from ..utils.logger import Logger
from ..utils.utils import check_nan, resolve_callable


def latest_checkpoint(log_dir: str | None) -> str | None:
    """The ``model_<iteration>.pt`` with the highest iteration in ``log_dir``, or None."""
    if not log_dir or not os.path.isdir(log_dir):
        return None
    best, best_it = None, -1
    for name in os.listdir(log_dir):
        m = re.fullmatch(r"model_(\d+)\.pt", name)
        if m and int(m.group(1)) > best_it:
            best, best_it = os.path.join(log_dir, name), int(m.group(1))
    return best


class OnPolicyRunner:
    alg: PPO

    def __init__(self, env, train_cfg: dict, log_dir: str | None = None, device: str = "cpu") -> None:
        self.env = env
        self.cfg = train_cfg
        self.device = device
        self.gpu_session = None
        guard = self.cfg.get("device_guard")
        if guard and torch.device(device).type == "cuda":
            # opt-in: device checks and an exclusive per-GPU lock before anything touches the GPU
            from ..device import acquire_gpu

            self.gpu_session = acquire_gpu(torch.device(device).index or 0, **(guard if isinstance(guard, dict) else {}))
        self._configure_multi_gpu()
        obs = self.env.get_observations()
        alg_class = resolve_callable(self.cfg["algorithm"]["class_name"])
        self.alg = alg_class.construct_algorithm(obs, self.env, self.cfg, self.device)
        self.logger = Logger(
            log_dir=log_dir, cfg=self.cfg, env_cfg=self.env.cfg, num_envs=self.env.num_envs,
            is_distributed=self.is_distributed, gpu_world_size=self.gpu_world_size,
            gpu_global_rank=self.gpu_global_rank, device=self.device,
        )
        self.current_learning_iteration = 0
        self._rollout_graph = None
        from ..utils.timer import SectionTimer

        b200 = self.alg.b200_cfg if hasattr(self.alg, "b200_cfg") else {}
        self.section_timer = SectionTimer(b200.get("section_timing", False), self.device)

    # ---- training loop ------------------------------------------------------------------------------------------------
    def learn(self, num_learning_iterations: int, init_at_random_ep_len: bool = False) -> None:
        if init_at_random_ep_len:
            self.env.episode_length_buf = torch.randint_like(self.env.episode_length_buf,
                                                             high=int(self.env.max_episode_length))
        obs = self.env.get_observations().to(self.device)
        self.alg.train_mode()
        if self.is_distributed:
            print(f"Synchronizing parameters for rank {self.gpu_global_rank}...")
            self.alg.broadcast_parameters()
        self.logger.init_logging_writer()
        start_it = self.current_learning_iteration
        total_it = start_it + num_learning_iterations
        try:
            timer = self.section_timer
            for it in range(start_it, total_it):
                t0 = time.time()
                with torch.inference_mode():
                    with timer.section("rollout"):
                        obs = self.rollout(obs)
                    t1 = time.time()
                    collect_time = t1 - t0
                    with timer.section("returns"):
                        self.alg.compute_returns(obs)
                with timer.section("update"):
                    loss_dict = self.alg.update()
                learn_time = time.time() - t1
                self.current_learning_iteration = it
                self.logger.log(
                    it=it, start_it=start_it, total_it=total_it, collect_time=collect_time, learn_time=learn_time,
                    loss_dict=loss_dict, learning_rate=self.alg.learning_rate,
                    action_std=self._action_std(),
                    rnd_weight=self.alg.rnd.weight if self.cfg["algorithm"].get("rnd_cfg") else None,
                    sections=timer.resolve() if timer.enabled else None,
                )
                if self.logger.writer is not None and it % self.cfg["save_interval"] == 0:
                    self.save(os.path.join(self.logger.log_dir, f"model_{it}.pt"))
            if self.logger.writer is not None:
                self.save(os.path.join(self.logger.log_dir, f"model_{self.current_learning_iteration}.pt"))
        except BaseException:
            self.logger.abort_logging_writer()
            raise
        self.logger.stop_logging_writer()

    def rollout(self, obs):
        """Collect ``num_steps_per_env`` transitions; returns the observations after the last step."""
        engine = getattr(self.alg, "engine", None)
        if engine is not None and engine.can_capture_rollout(self.env, self.cfg):
            return engine.run_captured_rollout(self.env, self.logger, self.cfg)
        check = self.cfg.get("check_for_nan", True)
        use_rnd = bool(self.cfg["algorithm"].get("rnd_cfg"))
        # a graph-capturable environment rewrites its observation tensors in place every step, while the PyTorch path
        # keeps a reference to the observations it acted on until the next step is stored (as rsl_rl does): give it a
        # copy. The fused engines copy observations into their own buffers and need none.
        copy_obs = engine is None and bool(getattr(self.env, "graph_capturable", False))
        for _ in range(self.cfg["num_steps_per_env"]):
            actions = self.alg.act(obs.clone() if copy_obs else obs)
            obs, rewards, dones, extras = self.env.step(actions.to(self.env.device))
            if check and engine is None:
                check_nan(obs, rewards, dones)
            obs, rewards, dones = obs.to(self.device), rewards.to(self.device), dones.to(self.device)
            if check and engine is not None:
                engine.check_finite(obs, rewards)
            self.alg.process_env_step(obs, rewards, dones, extras)
            intrinsic = self.alg.intrinsic_rewards if use_rnd else None
            self.logger.process_env_step(rewards, dones, extras, intrinsic)
        if check and engine is not None:
            engine.raise_if_nonfinite()
        return obs

    def _action_std(self) -> torch.Tensor:
        engine = getattr(self.alg, "engine", None)
        if engine is not None and hasattr(engine, "action_std"):
            return engine.action_std()
        policy = self.alg.get_policy()
        if getattr(policy, "distribution", None) is None or not policy.distribution.ready:
            return torch.zeros(1)
        return policy.output_std

    # ---- checkpoints ----------------------------------------------------------------------------------------------------
    def save(self, path: str, infos: dict | None = None) -> None:
        saved = self.alg.save()
        saved["iter"] = self.current_learning_iteration
        saved["infos"] = infos
        torch.save(saved, path)
        self.logger.save_model(path, self.current_learning_iteration)

    def load(self, path: str, load_cfg: dict | None = None, strict: bool = True,
             map_location: str | None = None) -> dict:
        loaded = torch.load(path, weights_only=False, map_location=map_location)
        if self.alg.load(loaded, load_cfg, strict):
            self.current_learning_iteration = loaded["iter"]
        return loaded.get("infos")

    def resume_latest(self, log_dir: str | None = None, **load_kwargs) -> str | None:
        """Load the newest ``model_<iteration>.pt`` of ``log_dir`` (default: this run's log folder) if there is one:
        the recovery path after a failed job (``python -m tt_rsl_rl_b200.launch --retries``). Returns the path."""
        path = latest_checkpoint(log_dir or self.logger.log_dir)
        if path is not None:
            self.load(path, **load_kwargs)
        return path

    def get_inference_policy(self, device: str | None = None):
        self.alg.eval_mode()
        return self.alg.get_policy().to(device)

    def export_policy_to_jit(self, path: str, filename: str = "policy.pt") -> None:
        model = self.alg.get_policy().as_jit()
        model.to("cpu")
        os.makedirs(path, exist_ok=True)
        torch.jit.script(model).save(os.path.join(path, filename))

    def export_policy_to_onnx(self, path: str, filename: str = "policy.onnx", verbose: bool = False) -> None:
        model = self.alg.get_policy().as_onnx()
        model.to("cpu")
        model.eval()
        os.makedirs(path, exist_ok=True)
        torch.onnx.export(model, model.get_dummy_inputs(), os.path.join(path, filename), export_params=True,
                          opset_version=18, verbose=verbose, input_names=model.input_names,
                          output_names=model.output_names)

    def add_git_repo_to_log(self, repo_file_path: str) -> None:
        self.logger.git_status_repos.append(repo_file_path)

    # ---- distributed setup ----------------------------------------------------------------------------------------------
    def _configure_multi_gpu(self) -> None:
        self.gpu_world_size = int(os.getenv("WORLD_SIZE", "1"))
        self.is_distributed = self.gpu_world_size > 1
        if not self.is_distributed:
            self.gpu_local_rank = 0
            self.gpu_global_rank = 0
            self.cfg["multi_gpu"] = None
            return
        self.gpu_local_rank = int(os.getenv("LOCAL_RANK", "0"))
        self.gpu_global_rank = int(os.getenv("RANK", "0"))
        self.cfg["multi_gpu"] = {
            "global_rank": self.gpu_global_rank,
            "local_rank": self.gpu_local_rank,
            "world_size": self.gpu_world_size,
        }
        is_cuda = torch.device(self.device).type == "cuda"
        if is_cuda and self.device != f"cuda:{self.gpu_local_rank}":
            raise ValueError(
                f"Device '{self.device}' does not match expected device for local rank '{self.gpu_local_rank}'."
            )
        if self.gpu_local_rank >= self.gpu_world_size:
            raise ValueError(
                f"Local rank '{self.gpu_local_rank}' is greater than or equal to world size '{self.gpu_world_size}'."
            )
        if self.gpu_global_rank >= self.gpu_world_size:
            raise ValueError(
                f"Global rank '{self.gpu_global_rank}' is greater than or equal to world size '{self.gpu_world_size}'."
            )
        if not torch.distributed.is_initialized():
            backend = "nccl" if is_cuda else "gloo"
            kwargs = {}
            if is_cuda:
                kwargs["device_id"] = torch.device(self.device)
            torch.distributed.init_process_group(backend=backend, rank=self.gpu_global_rank,
                                                 world_size=self.gpu_world_size, **kwargs)
        if is_cuda:
            torch.cuda.set_device(self.gpu_local_rank)
