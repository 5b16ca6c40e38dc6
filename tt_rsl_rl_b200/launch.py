"""Job launcher: lock the selected GPUs, record the job, run it (one process per GPU through ``torch.distributed.run``
on 127.0.0.1) under a time limit, and stop it cleanly.

::

    python -m tt_rsl_rl_b200.launch --gpus 0,1 --timeout 3600 --tag ppo -- train.py --task x
    python -m tt_rsl_rl_b200.launch --nproc 2 --timeout 60 -- test_gloo.py   # host only (no GPU selected)
    python -m tt_rsl_rl_b200.launch --list
    python -m tt_rsl_rl_b200.launch --stop-mine [--tag ppo]

What it does:

* ``--gpus``: ``CUDA_VISIBLE_DEVICES`` is set to the list, and every listed GPU's lock (the same lock file that
  :func:`tt_rsl_rl_b200.device.open_gpu` takes) is held for the whole job; a GPU that another job holds is refused
  (exit code 3) before anything starts. The job learns which locks its launcher holds from
  ``TT_RSL_RL_GPU_LOCKS_HELD``.
* the job runs in its own process group. At the time limit the group gets SIGINT (Python raises KeyboardInterrupt,
  so ``finally`` blocks release graphs and process groups), then SIGKILL after ``--grace`` seconds; the exit code is
  then 124, as for ``timeout``. SIGINT / SIGTERM sent to the launcher are passed on the same way.
* a record ``<run dir>/<tag>-<pid>.json`` (launcher PID, process group, GPUs, command, attempt, start time) exists
  while the job runs; ``--list`` prints the records and the lock holders, ``--stop-mine`` stops the recorded process
  groups of this user (exact group IDs from the records, never a name pattern).
* ``--retries N`` restarts a job that failed (not one that hit the limit or was stopped) with its GPUs still locked;
  the job reads its attempt number from ``TT_RSL_RL_ATTEMPT`` and resumes from its newest checkpoint.

The reference plugin's job wrapper has the same roles for Tenstorrent trays (``scripts/tt_run.sh``: lock, PID
record, device isolation, ``timeout`` with SIGINT then SIGKILL; ``scripts/kill_my_jobs.sh``).
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import socket
import subprocess
import sys
import time

from .device import LOCKS_HELD_ENV, DeviceGuardError, GpuLock, default_lock_dir, lock_path

RUN_DIR_ENV = "TT_RSL_RL_RUN_DIR"
ATTEMPT_ENV = "TT_RSL_RL_ATTEMPT"
EXIT_REFUSED = 3
EXIT_TIMEOUT = 124


def default_run_dir() -> str:
    return os.environ.get(RUN_DIR_ENV) or os.path.join(default_lock_dir(), "jobs")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def build_command(script: list[str], nproc: int, master_port: int, torchrun: bool = True) -> list[str]:
    """The child command: ``torch.distributed.run`` on one node at 127.0.0.1, or the script alone."""
    if not torchrun:
        return [sys.executable, *script]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
            "--master-addr=127.0.0.1", f"--master-port={master_port}", *script]


def _parse_gpus(text: str | None) -> list[int]:
    if not text:
        return []
    gpus = [int(g) for g in text.split(",") if g.strip()]
    if len(set(gpus)) != len(gpus):
        raise ValueError(f"--gpus lists a GPU twice: {text}")
    return gpus


def _signal_group(pgid: int, sig: int) -> None:
    try:
        os.killpg(pgid, sig)
    except ProcessLookupError:
        pass


def _supervise(cmd: list[str], child_env: dict, *, tag: str, gpus: list[int], record: str, timeout: float | None,
               grace: float, attempt: int) -> tuple[int, str]:
    """Run ``cmd`` in its own process group under the time limit; returns (exit code, "done" | "timeout" |
    "stopping")."""
    proc = subprocess.Popen(cmd, env=child_env, start_new_session=True)
    pgid = proc.pid  # a new session: the child leads its own process group
    with open(record, "w") as f:
        json.dump({"tag": tag, "launcher_pid": os.getpid(), "pgid": pgid, "uid": os.getuid(), "gpus": gpus,
                   "command": cmd, "attempt": attempt, "start": time.time()}, f)
    stopping = {"sig": None}

    def forward(signum, _frame):
        stopping["sig"] = signum
        _signal_group(pgid, signal.SIGINT)

    old = {s: signal.signal(s, forward) for s in (signal.SIGINT, signal.SIGTERM)}
    state, kill_at = "running", None  # running -> "timeout" (limit reached) or "stopping" (signal received)
    try:
        deadline = None if timeout is None else time.monotonic() + timeout
        while proc.poll() is None:
            now = time.monotonic()
            if state == "running":
                if deadline is not None and now >= deadline:
                    state, kill_at = "timeout", now + grace
                    print(f"launch: {tag} reached its limit of {timeout:g} s; interrupting", file=sys.stderr)
                    _signal_group(pgid, signal.SIGINT)
                elif stopping["sig"] is not None:
                    state, kill_at = "stopping", now + grace  # the handler already sent the interrupt
            elif now >= kill_at:
                print(f"launch: {tag} still running {grace:g} s after the interrupt; killing", file=sys.stderr)
                _signal_group(pgid, signal.SIGKILL)
                break
            time.sleep(0.05)
        rc = proc.wait()
        _signal_group(pgid, signal.SIGKILL)  # stragglers left in the group
    finally:
        for s, h in old.items():
            signal.signal(s, h)
    if state == "running" and stopping["sig"] is not None:
        state = "stopping"
    return rc, ("done" if state == "running" else state)


def run_job(script: list[str], *, gpus: list[int], nproc: int | None = None, timeout: float | None = None,
            grace: float = 30.0, tag: str = "job", run_dir: str | None = None, lock_dir: str | None = None,
            master_port: int | None = None, torchrun: bool = True, env: dict | None = None,
            retries: int = 0) -> int:
    """Run one job as described in the module docstring and return its exit code.

    ``retries`` restarts a job that failed (non-zero exit, neither the time limit nor a stop request) up to that many
    times, with the GPUs still locked; the job sees its attempt number in ``TT_RSL_RL_ATTEMPT`` and can resume from
    its newest checkpoint (``OnPolicyRunner.resume_latest``). The time limit applies to each attempt."""
    nproc = nproc or max(len(gpus), 1)
    if gpus and nproc != len(gpus):
        raise ValueError(f"{len(gpus)} GPUs selected but {nproc} processes requested")
    lock_dir = lock_dir or default_lock_dir()
    run_dir = run_dir or default_run_dir()
    locks: list[GpuLock] = []
    try:
        for g in gpus:
            lk = GpuLock(lock_path(g, lock_dir))
            lk.acquire()
            locks.append(lk)
    except DeviceGuardError as exc:
        for lk in locks:
            lk.release()
        print(f"launch: refused: {exc}", file=sys.stderr)
        return EXIT_REFUSED
    child_env = dict(os.environ if env is None else env)
    if gpus:
        child_env["CUDA_VISIBLE_DEVICES"] = ",".join(str(g) for g in gpus)
        child_env[LOCKS_HELD_ENV] = ",".join(str(g) for g in gpus)
    os.makedirs(run_dir, exist_ok=True)
    record = os.path.join(run_dir, f"{tag}-{os.getpid()}.json")
    try:
        for attempt in range(retries + 1):
            child_env[ATTEMPT_ENV] = str(attempt)
            cmd = build_command(script, nproc, master_port or free_port(), torchrun)
            rc, how = _supervise(cmd, child_env, tag=tag, gpus=gpus, record=record, timeout=timeout, grace=grace,
                                 attempt=attempt)
            if how == "timeout":
                return EXIT_TIMEOUT
            if rc == 0 or how == "stopping" or attempt == retries:
                return rc
            print(f"launch: {tag} attempt {attempt} failed with exit code {rc}; restarting", file=sys.stderr)
        return rc
    finally:
        for lk in locks:
            lk.release()
        try:
            os.remove(record)
        except OSError:
            pass


def list_jobs(run_dir: str | None = None) -> list[dict]:
    """Records of running jobs (stale records, whose launcher is gone, are dropped)."""
    run_dir = run_dir or default_run_dir()
    out = []
    if not os.path.isdir(run_dir):
        return out
    for name in sorted(os.listdir(run_dir)):
        if not name.endswith(".json"):
            continue
        path = os.path.join(run_dir, name)
        try:
            with open(path) as f:
                rec = json.load(f)
            try:
                os.kill(rec["launcher_pid"], 0)
            except PermissionError:
                pass  # another user's live launcher
        except (OSError, ValueError, KeyError):
            try:
                os.remove(path)
            except OSError:
                pass
            continue
        out.append(rec)
    return out


def lock_holders(lock_dir: str | None = None) -> dict[str, str]:
    lock_dir = lock_dir or default_lock_dir()
    if not os.path.isdir(lock_dir):
        return {}
    return {n: GpuLock.holder(os.path.join(lock_dir, n)) for n in sorted(os.listdir(lock_dir)) if n.endswith(".lock")}


def stop_mine(tag: str | None = None, run_dir: str | None = None, sig: int = signal.SIGINT) -> list[int]:
    """Send ``sig`` to the process group of every recorded job of this user (optionally only ``tag``)."""
    stopped = []
    for rec in list_jobs(run_dir):
        if rec.get("uid") != os.getuid() or (tag is not None and rec.get("tag") != tag):
            continue
        _signal_group(int(rec["pgid"]), sig)
        stopped.append(int(rec["pgid"]))
    return stopped


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    script: list[str] = []
    if "--" in argv:
        i = argv.index("--")
        argv, script = argv[:i], argv[i + 1:]
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", default=None, help="comma-separated GPU indices (one process each)")
    ap.add_argument("--nproc", type=int, default=None, help="processes when no GPU is selected")
    ap.add_argument("--timeout", type=float, default=None, help="seconds before the job is interrupted")
    ap.add_argument("--grace", type=float, default=30.0, help="seconds between the interrupt and SIGKILL")
    ap.add_argument("--retries", type=int, default=0, help="restart a failed job up to this many times")
    ap.add_argument("--tag", default="job")
    ap.add_argument("--master-port", type=int, default=None)
    ap.add_argument("--no-torchrun", action="store_true", help="run the script directly (one process)")
    ap.add_argument("--run-dir", default=None)
    ap.add_argument("--lock-dir", default=None)
    ap.add_argument("--list", action="store_true", help="print the running jobs and the GPU lock holders")
    ap.add_argument("--stop-mine", action="store_true", help="interrupt this user's recorded jobs")
    args = ap.parse_args(argv)
    if args.list:
        print(json.dumps({"jobs": list_jobs(args.run_dir), "locks": lock_holders(args.lock_dir)}, indent=1))
        return 0
    if args.stop_mine:
        print(json.dumps({"stopped_process_groups": stop_mine(args.tag if args.tag != "job" else None,
                                                               args.run_dir)}))
        return 0
    if not script:
        ap.error("give the job after '--'")
    return run_job(script, gpus=_parse_gpus(args.gpus), nproc=args.nproc, timeout=args.timeout, grace=args.grace,
                   tag=args.tag, run_dir=args.run_dir, lock_dir=args.lock_dir, master_port=args.master_port,
                   torchrun=not args.no_torchrun, retries=args.retries)


if __name__ == "__main__":
    sys.exit(main())
