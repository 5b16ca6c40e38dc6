"""Neptune writer (``rsl_rl/utils/neptune_log_writer.py``): every scalar goes to TensorBoard files in the run folder
and to a Neptune run; configurations, checkpoints and files are uploaded. ``neptune`` is imported on construction.

Kept as upstream has them: the project ``$NEPTUNE_USERNAME/<project_name>`` with the token from
``NEPTUNE_API_TOKEN`` (a clear error when either is missing), the run's ``log_dir`` entry, the keys ``train_cfg`` /
``env_cfg``, ``model/saved_model_<it>`` and ``git_diff/<name>``, and the renaming of time-indexed tags.
"""

from __future__ import annotations

import os
import pathlib

from torch.utils.tensorboard import SummaryWriter

from .log_writer import LogWriter
from .wandb_log_writer import env_cfg_dict

_NAME_MAP = {"Train/mean_reward/time": "Train/mean_reward_time",
             "Train/mean_episode_length/time": "Train/mean_episode_length_time"}


class NeptuneLogWriter(SummaryWriter, LogWriter):
    def __init__(self, log_dir: str, project_name: str | None = None, **kwargs) -> None:
        try:
            import neptune  # type: ignore
        except ImportError as exc:
            raise ModuleNotFoundError("NeptuneLogWriter requires the 'neptune' package") from exc
        token, user = os.environ.get("NEPTUNE_API_TOKEN"), os.environ.get("NEPTUNE_USERNAME")
        if token is None:
            raise KeyError("NEPTUNE_API_TOKEN is not set: export NEPTUNE_API_TOKEN=<your token>")
        if user is None:
            raise KeyError("NEPTUNE_USERNAME is not set: export NEPTUNE_USERNAME=<your user name>")
        super().__init__(log_dir, flush_secs=10)
        self.run = neptune.init_run(project=f"{user}/{project_name}", api_token=token, **kwargs)
        self.run["log_dir"].log(os.path.split(log_dir.rstrip("/"))[-1])

    def add_scalar(self, tag: str, scalar_value: float, global_step: int | None = None, walltime: float | None = None,
                   new_style: bool = False) -> None:
        super().add_scalar(tag, scalar_value, global_step=global_step, walltime=walltime, new_style=new_style)
        self.run[_NAME_MAP.get(tag, tag)].log(scalar_value, step=global_step)

    def store_config(self, env_cfg, train_cfg: dict) -> None:
        self.run["train_cfg"] = train_cfg
        self.run["env_cfg"] = env_cfg_dict(env_cfg)

    def save_model(self, model_path: str, it: int) -> None:
        self.run[f"model/saved_model_{it}"].upload(model_path)

    def save_file(self, path: str) -> None:
        self.run["git_diff/" + os.path.basename(path).split(".")[0]].upload(path)

    def save_video(self, video: pathlib.Path, it: int) -> None:
        self.run[f"videos/{pathlib.Path(video).name}"].upload(str(video))

    def stop(self) -> None:
        self.close()
        self.run.stop()
