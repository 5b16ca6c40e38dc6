"""The scripts under ``examples/`` run end to end on the CPU (tiny sizes): train, evaluate + export, distil."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXAMPLES = os.path.join(ROOT, "examples", "tracking12")


def _run(script: str, *args: str, cwd: str) -> str:
    out = subprocess.run([sys.executable, os.path.join(EXAMPLES, script), "--device", "cpu", *args], cwd=cwd,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout


@pytest.fixture(scope="module")
def ppo_run(tmp_path_factory):
    work = tmp_path_factory.mktemp("examples")
    log_dir = str(work / "ppo")
    _run("train.py", "--envs", "32", "--iterations", "3", "--save-interval", "2", "--log-dir", log_dir, cwd=str(work))
    return work, log_dir


def test_train_writes_checkpoints_and_resumes(ppo_run):
    work, log_dir = ppo_run
    assert {"model_0.pt", "model_2.pt", "metrics.csv", "config.json"} <= set(os.listdir(log_dir))
    # the checkpoint of iteration 2 restarts at iteration 2 (rsl_rl's numbering): two more iterations end at 3
    out = _run("train.py", "--envs", "32", "--iterations", "2", "--log-dir", log_dir, cwd=str(work))
    assert "resuming from" in out and "model_2.pt" in out
    assert "model_3.pt" in os.listdir(log_dir)


def test_play_evaluates_and_exports(ppo_run):
    work, log_dir = ppo_run
    out = _run("play.py", "--envs", "16", "--steps", "50", "--log-dir", log_dir, "--export", str(work / "exp"),
               cwd=str(work))
    stats = json.loads(out.strip().splitlines()[-1])
    assert stats["checkpoint"].endswith(".pt") and os.path.isfile(stats["exported"])


def test_distill_from_the_ppo_checkpoint(ppo_run):
    work, log_dir = ppo_run
    student_dir = str(work / "student")
    _run("distill.py", "--envs", "32", "--iterations", "2", "--teacher-dir", log_dir, "--log-dir", student_dir,
         cwd=str(work))
    assert "model_1.pt" in os.listdir(student_dir)
