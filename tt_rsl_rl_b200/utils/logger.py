"""Training logger with rsl_rl's metrics and console output (``rsl_rl/utils/logger.py``).

Difference in mechanism (not in what is logged): episode bookkeeping stays on the device. Every environment step only
enqueues device work (running episode sums, a per-step record of finished episodes), so the rollout loop has no host
synchronisation and can be captured in a CUDA graph. Finished episodes are compacted and copied to the host once per
iteration in :meth:`Logger.log`, where the last-100-episode buffers are updated exactly as upstream's per-step
``deque.extend`` would have left them.
"""

from __future__ import annotations

import datetime
import os
import pathlib
import statistics
import warnings
from collections import deque

import torch

from .log_writer import LogWriter
from .utils import resolve_class


class Logger:
    def __init__(self, log_dir: str | None, cfg: dict, env_cfg, num_envs: int, is_distributed: bool,
                 gpu_world_size: int, gpu_global_rank: int, device: str, num_steps_per_env: int | None = None) -> None:
        import tt_rsl_rl_b200

        self.log_dir = log_dir
        self.cfg = cfg
        self.env_cfg = env_cfg
        self.num_envs = num_envs
        self.gpu_world_size = gpu_world_size
        self.device = device
        self.git_status_repos = [tt_rsl_rl_b200.__file__]
        self.tot_timesteps = 0
        self.tot_time = 0.0
        self.writer = None
        self.uploaded_videos: set[pathlib.Path] = set()
        self.disable_logs = is_distributed and gpu_global_rank != 0
        self.use_rnd = bool(cfg["algorithm"].get("rnd_cfg"))
        T = num_steps_per_env or cfg["num_steps_per_env"]
        self.rewbuffer: deque = deque(maxlen=100)
        self.lenbuffer: deque = deque(maxlen=100)
        self.erewbuffer: deque = deque(maxlen=100)
        self.irewbuffer: deque = deque(maxlen=100)
        dev = device
        self.cur_reward_sum = torch.zeros(num_envs, device=dev)
        self.cur_episode_length = torch.zeros(num_envs, device=dev)
        self.cur_ereward_sum = torch.zeros(num_envs, device=dev)
        self.cur_ireward_sum = torch.zeros(num_envs, device=dev)
        # per-step records of finished episodes, compacted once per iteration
        self._cap = T
        self._fin_done = torch.zeros(T, num_envs, dtype=torch.bool, device=dev)
        self._fin_rew = torch.zeros(T, num_envs, device=dev)
        self._fin_len = torch.zeros(T, num_envs, device=dev)
        self._fin_erew = torch.zeros(T, num_envs, device=dev) if self.use_rnd else None
        self._fin_irew = torch.zeros(T, num_envs, device=dev) if self.use_rnd else None
        self._step = 0
        self._extras_sum: dict[str, torch.Tensor] = {}
        self._extras_cnt: dict[str, int] = {}
        self._extras_order: list[str] = []
        # per-step values of eager steps (none are kept while a rollout is being captured into a CUDA graph): their
        # mean is taken over the concatenation, in one reduction, as rsl_rl does; replayed rollouts use the sums
        self._extras_vals: dict[str, list[torch.Tensor]] = {}

    # ---- writer lifecycle ----------------------------------------------------------------------------------------------
    def init_logging_writer(self) -> None:
        if self.log_dir is not None and not self.disable_logs:
            logger_cfg = self.cfg.get("logger", "tensorboard")
            name = logger_cfg if isinstance(logger_cfg, str) else logger_cfg["class_name"]
            if isinstance(logger_cfg, str) and name in ("wandb", "neptune"):
                warnings.warn(f"cfg['logger'] = '{name}' is deprecated; use the dict form with 'class_name'.",
                              DeprecationWarning, stacklevel=2)
                cls_name = "WandbLogWriter" if name == "wandb" else "NeptuneLogWriter"
                logger_cfg = {"class_name": cls_name, "project_name": self.cfg.get(f"{name}_project")}
                name = cls_name
            if name == "tensorboard":
                from torch.utils.tensorboard import SummaryWriter

                self.writer = SummaryWriter(log_dir=self.log_dir, flush_secs=10)
            else:
                cls, kwargs = resolve_class(logger_cfg)
                self.writer = cls(log_dir=self.log_dir, **kwargs)
        else:
            self.writer = None
        files = self._store_code_state()
        if isinstance(self.writer, LogWriter):
            self.writer.store_config(self.env_cfg, self.cfg)
            for path in files:
                self.writer.save_file(path)

    # ---- per step (device work only) ---------------------------------------------------------------------------------
    def process_env_step(self, rewards: torch.Tensor, dones: torch.Tensor, extras: dict,
                         intrinsic_rewards: torch.Tensor | None = None) -> None:
        if self.writer is None:
            return
        info = extras.get("episode", extras.get("log"))
        if info:
            for key, value in info.items():
                if key not in self._extras_sum:
                    with torch.inference_mode(False):  # a normal tensor: it is also reset outside inference mode
                        self._extras_sum[key] = torch.zeros((), device=self.device)
                    self._extras_cnt[key] = 0
                if key not in self._extras_order:  # keys seen in this iteration, in order of first appearance
                    self._extras_order.append(key)
                v = value if isinstance(value, torch.Tensor) else torch.tensor(float(value))
                v = v.to(self.device, torch.float32).reshape(-1)
                self._extras_sum[key] += v.sum()
                self._extras_cnt[key] += v.numel()
                if not (torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()):
                    self._extras_vals.setdefault(key, []).append(v.clone())
        rewards = rewards.to(self.device).view(-1)
        if intrinsic_rewards is not None:
            self.cur_ereward_sum += rewards
            self.cur_ireward_sum += intrinsic_rewards
            self.cur_reward_sum += rewards + intrinsic_rewards
        else:
            self.cur_reward_sum += rewards
        self.cur_episode_length += 1
        done = dones.to(self.device).view(-1) > 0
        if self._step >= self._cap:
            self._flush_finished()
        t = self._step
        self._fin_done[t].copy_(done)
        self._fin_rew[t].copy_(self.cur_reward_sum)
        self._fin_len[t].copy_(self.cur_episode_length)
        keep = (~done).float()
        self.cur_reward_sum *= keep
        self.cur_episode_length *= keep
        if intrinsic_rewards is not None and self._fin_erew is not None:
            self._fin_erew[t].copy_(self.cur_ereward_sum)
            self._fin_irew[t].copy_(self.cur_ireward_sum)
            self.cur_ereward_sum *= keep
            self.cur_ireward_sum *= keep
        self._step += 1

    def _flush_finished(self) -> None:
        """Move finished episodes (in step order, env order within a step) into the 100-episode buffers."""
        n = self._step
        if n == 0:
            return
        mask = self._fin_done[:n]
        count = int(mask.sum())
        if count > 0:
            take = min(count, 100)

            def last(x: torch.Tensor) -> list[float]:
                return x[:n][mask][-take:].cpu().tolist()

            self.rewbuffer.extend(last(self._fin_rew))
            self.lenbuffer.extend(last(self._fin_len))
            if self._fin_erew is not None:
                self.erewbuffer.extend(last(self._fin_erew))
                self.irewbuffer.extend(last(self._fin_irew))
        self._fin_done[:n] = False
        self._step = 0

    # ---- host-side state (for CUDA-graph capture of the rollout) ----------------------------------------------------
    def host_state(self) -> tuple:
        """Snapshot of the host-side counters that :meth:`process_env_step` advances."""
        return self._step, dict(self._extras_cnt), list(self._extras_order)

    def set_host_state(self, state: tuple) -> None:
        self._step, cnt, order = state
        self._extras_cnt = dict(cnt)
        self._extras_order = list(order)

    def advance_host_state(self, before: tuple, after: tuple) -> None:
        """Apply the counter changes of one captured rollout (``before`` -> ``after``) after a graph replay."""
        self._step += after[0] - before[0]
        for key, n in after[1].items():
            self._extras_cnt[key] = self._extras_cnt.get(key, 0) + n - before[1].get(key, 0)
        for key in after[2]:
            if key not in self._extras_order:
                self._extras_order.append(key)

    # ---- per iteration -------------------------------------------------------------------------------------------------
    def log(self, it: int, start_it: int, total_it: int, collect_time: float, learn_time: float, loss_dict: dict,
            learning_rate: float, action_std: torch.Tensor, rnd_weight: float | None, print_minimal: bool = False,
            width: int = 80, pad: int = 40, sections: dict[str, float] | None = None) -> None:
        if self.writer is None:
            return
        self._flush_finished()
        collection_size = self.cfg["num_steps_per_env"] * self.num_envs * self.gpu_world_size
        iteration_time = collect_time + learn_time
        self.tot_timesteps += collection_size
        self.tot_time += iteration_time
        extras_string = ""
        for key in self._extras_order:
            vals = self._extras_vals.get(key)
            if vals and sum(v.numel() for v in vals) == self._extras_cnt[key]:  # every step of the iteration was eager
                value = torch.mean(torch.cat(vals)).item()
            else:
                value = (self._extras_sum[key] / max(1, self._extras_cnt[key])).item()
            if "/" in key:
                self.writer.add_scalar(key, value, it)
                extras_string += f"""{f"{key}:":>{pad}} {value:.4f}\n"""
            else:
                self.writer.add_scalar("Episode/" + key, value, it)
                extras_string += f"""{f"Mean episode {key}:":>{pad}} {value:.4f}\n"""
        for v in self._extras_sum.values():
            v.zero_()  # persistent accumulators (captured rollouts add into them)
        self._extras_cnt = {k: 0 for k in self._extras_cnt}
        self._extras_order.clear()
        self._extras_vals.clear()
        for key, value in loss_dict.items():
            self.writer.add_scalar(f"Loss/{key}", value, it)
        self.writer.add_scalar("Loss/learning_rate", learning_rate, it)
        mean_std = action_std.float().mean().item()
        self.writer.add_scalar("Policy/mean_std", mean_std, it)
        fps = int(collection_size / max(iteration_time, 1e-9))
        self.writer.add_scalar("Perf/total_fps", fps, it)
        self.writer.add_scalar("Perf/collection_time", collect_time, it)
        self.writer.add_scalar("Perf/learning_time", learn_time, it)
        for name, ms in (sections or {}).items():
            self.writer.add_scalar(f"Perf/section_{name}_ms", ms, it)
        if len(self.rewbuffer) > 0:
            if self.use_rnd:
                self.writer.add_scalar("Rnd/mean_extrinsic_reward", statistics.mean(self.erewbuffer), it)
                self.writer.add_scalar("Rnd/mean_intrinsic_reward", statistics.mean(self.irewbuffer), it)
                self.writer.add_scalar("Rnd/weight", rnd_weight, it)
            self.writer.add_scalar("Train/mean_reward", statistics.mean(self.rewbuffer), it)
            self.writer.add_scalar("Train/mean_episode_length", statistics.mean(self.lenbuffer), it)
            if not isinstance(self.writer, LogWriter):
                self.writer.add_scalar("Train/mean_reward/time", statistics.mean(self.rewbuffer), int(self.tot_time))
                self.writer.add_scalar("Train/mean_episode_length/time", statistics.mean(self.lenbuffer),
                                       int(self.tot_time))
        s = f"""{"#" * width}\n"""
        s += f"""\033[1m{f" Learning iteration {it}/{total_it} ".center(width)}\033[0m \n\n"""
        run_name = self.cfg.get("run_name")
        s += f"""{"Run name:":>{pad}} {run_name}\n""" if run_name else ""
        s += (f"""{"Total steps:":>{pad}} {self.tot_timesteps} \n"""
              f"""{"Steps per second:":>{pad}} {fps:.0f} \n"""
              f"""{"Collection time:":>{pad}} {collect_time:.3f}s \n"""
              f"""{"Learning time:":>{pad}} {learn_time:.3f}s \n""")
        for name, ms in (sections or {}).items():
            s += f"""{f"Section {name}:":>{pad}} {ms:.3f}ms\n"""
        for key, value in loss_dict.items():
            s += f"""{f"Mean {key} loss:":>{pad}} {value:.4f}\n"""
        if len(self.rewbuffer) > 0:
            if self.use_rnd:
                s += f"""{"Mean extrinsic reward:":>{pad}} {statistics.mean(self.erewbuffer):.2f}\n"""
                s += f"""{"Mean intrinsic reward:":>{pad}} {statistics.mean(self.irewbuffer):.2f}\n"""
            s += f"""{"Mean reward:":>{pad}} {statistics.mean(self.rewbuffer):.2f}\n"""
            s += f"""{"Mean episode length:":>{pad}} {statistics.mean(self.lenbuffer):.2f}\n"""
        s += f"""{"Mean action std:":>{pad}} {mean_std:.2f}\n"""
        if not print_minimal:
            s += extras_string
        done_it = it + 1 - start_it
        eta = self.tot_time / done_it * (total_it - start_it - done_it)
        s += (f"""{"-" * width}\n"""
              f"""{"Iteration time:":>{pad}} {iteration_time:.2f}s\n"""
              f"""{"Time elapsed:":>{pad}} {datetime.timedelta(seconds=int(self.tot_time))}\n"""
              f"""{"ETA:":>{pad}} {datetime.timedelta(seconds=int(eta))}\n""")
        print(s)
        if isinstance(self.writer, LogWriter):
            for video in pathlib.Path(self.log_dir).rglob("*.mp4"):
                if video not in self.uploaded_videos:
                    self.writer.save_video(video, it)
                    self.uploaded_videos.add(video)

    def save_model(self, path: str, it: int) -> None:
        if isinstance(self.writer, LogWriter):
            self.writer.save_model(path, it)

    def stop_logging_writer(self) -> None:
        if isinstance(self.writer, LogWriter):
            self.writer.stop()

    def abort_logging_writer(self) -> None:
        if isinstance(self.writer, LogWriter):
            self.writer.abort()

    def _store_code_state(self) -> list[str]:
        """Write ``<log_dir>/git/<repo>.diff`` (commit, status, diff) for every registered repository."""
        files: list[str] = []
        if self.log_dir is None or self.disable_logs:
            return files
        git_dir = os.path.join(self.log_dir, "git")
        os.makedirs(git_dir, exist_ok=True)
        try:
            import git  # type: ignore
        except ImportError:
            return files
        for path in self.git_status_repos:
            try:
                repo = git.Repo(path, search_parent_directories=True)
                tree = repo.head.commit.tree
                sha = repo.head.commit.hexsha
            except Exception:
                print(f"Could not find git repository in {path}. Skipping.")
                continue
            name = pathlib.Path(repo.working_dir).name
            out = os.path.join(git_dir, f"{name}.diff")
            if os.path.isfile(out):
                continue
            print(f"Storing git diff for '{name}' in: {out}")
            with open(out, "x", encoding="utf-8") as f:
                f.write(f"--- git commit ---\n{sha}\n\n\n--- git status ---\n{repo.git.status()} \n\n\n"
                        f"--- git diff ---\n{repo.git.diff(tree)}")
            files.append(out)
        return files
