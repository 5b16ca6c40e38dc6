"""Pluggable logging back ends (``rsl_rl/utils/log_writer.py``): only :meth:`LogWriter.add_scalar` is required."""

from __future__ import annotations

import csv
import json
import os
import pathlib
from abc import ABC, abstractmethod


class LogWriter(ABC):
    @abstractmethod
    def add_scalar(self, tag: str, scalar_value: float, global_step: int) -> None:
        """Record one scalar."""

    def store_config(self, env_cfg: dict | object, train_cfg: dict) -> None:
        """Called once at the start of training."""

    def save_model(self, model_path: str, it: int) -> None:
        """Upload a checkpoint."""

    def save_file(self, path: str) -> None:
        """Upload a file."""

    def save_video(self, video: pathlib.Path, it: int) -> None:
        """Upload a video."""

    def stop(self) -> None:
        """Close the run."""

    def abort(self) -> None:
        """Close the run after an interruption (defaults to :meth:`stop`)."""
        self.stop()


class CsvLogWriter(LogWriter):
    """One CSV row per iteration (``metrics.csv``) plus ``config.json`` in ``log_dir`` (no external service)."""

    def __init__(self, log_dir: str, filename: str = "metrics.csv") -> None:
        self.log_dir = log_dir
        os.makedirs(log_dir, exist_ok=True)
        self.path = os.path.join(log_dir, filename)
        self._row: dict[str, float] = {}
        self._step: int | None = None
        self._columns: list[str] | None = None

    def add_scalar(self, tag: str, scalar_value: float, global_step: int) -> None:
        if self._step is not None and global_step != self._step:
            self._flush()
        self._step = global_step
        self._row[tag] = float(scalar_value)

    def _flush(self) -> None:
        if self._step is None:
            return
        row = {"iteration": self._step, **self._row}
        new = self._columns is None
        if new:
            self._columns = list(row)
        with open(self.path, "a", newline="") as f:
            w = csv.DictWriter(f, fieldnames=self._columns, extrasaction="ignore")
            if new:
                w.writeheader()
            w.writerow(row)
        self._row = {}

    def store_config(self, env_cfg: dict | object, train_cfg: dict) -> None:
        def default(o):
            return repr(o)

        with open(os.path.join(self.log_dir, "config.json"), "w") as f:
            json.dump({"env_cfg": env_cfg if isinstance(env_cfg, dict) else repr(env_cfg), "train_cfg": train_cfg}, f,
                      default=default, indent=2)

    def stop(self) -> None:
        self._flush()
        self._step = None
