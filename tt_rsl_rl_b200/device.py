"""Guarded opening of this process's GPU: the one place that selects the CUDA device for a training job.

:func:`open_gpu` runs these checks, in order, before anything touches the device:

1. at most one session per process;
2. the device index (argument, else ``LOCAL_RANK``, else 0) names a visible CUDA device;
3. the device is a Blackwell B200-class part (compute capability 10.0), the architecture the kernels are built for;
4. an exclusive per-GPU lock (``flock`` on ``<lock dir>/gpu<physical index>.lock``, holder PID written inside), so two
   jobs never share a GPU; skipped when the launcher (:mod:`tt_rsl_rl_b200.launch`) already holds it for this job
   (``TT_RSL_RL_GPU_LOCKS_HELD``);
5. at least ``min_free_bytes`` of device memory free;
6. the kernel extension loads (when ``require_extension``).

Only then is the device made current. :class:`GpuSession` runs its close hooks in reverse order (release CUDA graphs
and peer mappings before the context goes), synchronises, drops the lock and unregisters its ``atexit`` hook; closing
twice is a no-op. Every system call goes through :class:`Deps`, so the logic is tested on a host without a GPU.

The reference plugin guards its device the same way, for Tenstorrent meshes (``rsl_rl_tt/device.py:212-344``: one
guarded entry, ``Deps`` injection, close hooks, ``atexit``).
"""

from __future__ import annotations

import atexit
import fcntl
import os
import sys
import tempfile
from collections.abc import Callable, Mapping
from dataclasses import dataclass, field
from typing import Any

LOCK_DIR_ENV = "TT_RSL_RL_LOCK_DIR"
LOCKS_HELD_ENV = "TT_RSL_RL_GPU_LOCKS_HELD"
REQUIRED_CAPABILITY = (10, 0)


class DeviceGuardError(RuntimeError):
    """A device check failed; nothing (or nothing more) was opened."""


def default_lock_dir(environ: Mapping[str, str] | None = None) -> str:
    environ = os.environ if environ is None else environ
    return environ.get(LOCK_DIR_ENV) or os.path.join(tempfile.gettempdir(), "tt_rsl_rl_b200_locks")


def lock_path(physical_index: int, lock_dir: str) -> str:
    return os.path.join(lock_dir, f"gpu{physical_index}.lock")


def physical_index(local_index: int, environ: Mapping[str, str]) -> int | str:
    """The host's index of visible device ``local_index`` (``CUDA_VISIBLE_DEVICES`` remaps; UUID entries stay as
    given)."""
    visible = environ.get("CUDA_VISIBLE_DEVICES")
    if not visible:
        return local_index
    entries = [e.strip() for e in visible.split(",") if e.strip()]
    if local_index >= len(entries):
        return local_index
    e = entries[local_index]
    return int(e) if e.isdigit() else e


class GpuLock:
    """Exclusive, non-blocking ``flock`` on one GPU's lock file; the file holds the owner's PID."""

    def __init__(self, path: str) -> None:
        self.path = path
        self._fd: int | None = None

    @staticmethod
    def holder(path: str) -> str:
        try:
            with open(path) as f:
                return f.read().strip() or "unknown"
        except OSError:
            return "unknown"

    def acquire(self) -> None:
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        fd = os.open(self.path, os.O_RDWR | os.O_CREAT, 0o666)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX | fcntl.LOCK_NB)
        except BlockingIOError:
            os.close(fd)
            raise DeviceGuardError(f"GPU lock {self.path} is held by process {self.holder(self.path)}") from None
        os.ftruncate(fd, 0)
        os.write(fd, str(os.getpid()).encode())
        self._fd = fd

    def release(self) -> None:
        if self._fd is None:
            return
        try:
            os.ftruncate(self._fd, 0)
            fcntl.flock(self._fd, fcntl.LOCK_UN)
        finally:
            os.close(self._fd)
            self._fd = None

    @property
    def held(self) -> bool:
        return self._fd is not None


def _torch_capability(i: int) -> tuple[int, int]:
    import torch

    return tuple(torch.cuda.get_device_capability(i))


def _torch_mem_get_info(i: int) -> tuple[int, int]:
    import torch

    return tuple(torch.cuda.mem_get_info(i))


def _load_extension() -> Any:
    from .ops import ext

    return ext()


def _cuda_available() -> bool:
    import torch

    return torch.cuda.is_available()


def _device_count() -> int:
    import torch

    return torch.cuda.device_count()


def _set_device(i: int) -> None:
    import torch

    torch.cuda.set_device(i)


def _synchronize(i: int) -> None:
    import torch

    torch.cuda.synchronize(i)


@dataclass
class Deps:
    """System calls of the guard (replaced by fakes in host tests)."""

    environ: Mapping[str, str] = field(default_factory=lambda: os.environ)
    cuda_available: Callable[[], bool] = _cuda_available
    device_count: Callable[[], int] = _device_count
    capability: Callable[[int], tuple[int, int]] = _torch_capability
    mem_get_info: Callable[[int], tuple[int, int]] = _torch_mem_get_info
    load_extension: Callable[[], Any] = _load_extension
    set_device: Callable[[int], None] = _set_device
    synchronize: Callable[[int], None] = _synchronize


_ACTIVE: GpuSession | None = None


class GpuSession:
    """This process's open GPU. Context manager; :meth:`close` is idempotent and also runs at interpreter exit."""

    def __init__(self, index: int, physical: int | str, lock: GpuLock | None, deps: Deps) -> None:
        self.index = index
        self.physical_index = physical
        self.device = f"cuda:{index}"
        self._lock = lock
        self._deps = deps
        self._hooks: list[Callable[[], None]] = []
        self.closed = False

    def add_close_hook(self, hook: Callable[[], None]) -> None:
        """Run ``hook()`` before the session closes (hooks run in reverse order of registration)."""
        self._hooks.append(hook)

    @property
    def lock_held(self) -> bool:
        return self._lock is not None and self._lock.held

    def close(self) -> None:
        global _ACTIVE
        if self.closed:
            return
        self.closed = True
        error: BaseException | None = None
        for hook in reversed(self._hooks):
            try:
                hook()
            except BaseException as exc:  # the remaining hooks and the release still run
                print(f"tt_rsl_rl_b200.device: close hook failed: {exc!r}", file=sys.stderr)
                error = error or exc
        self._hooks.clear()
        try:
            self._deps.synchronize(self.index)
        except BaseException as exc:
            error = error or exc
        if self._lock is not None:
            self._lock.release()
        if _ACTIVE is self:
            _ACTIVE = None
        atexit.unregister(self.close)
        if error is not None:
            raise error

    def __enter__(self) -> GpuSession:
        return self

    def __exit__(self, *exc_info) -> None:
        self.close()


def _held_by_launcher(physical: int | str, environ: Mapping[str, str]) -> bool:
    held = environ.get(LOCKS_HELD_ENV, "")
    return str(physical) in {h.strip() for h in held.split(",") if h.strip()}


def open_gpu(local_index: int | None = None, *, lock: bool = True, lock_dir: str | None = None,
             min_free_bytes: int = 0, require_capability: tuple[int, int] | None = REQUIRED_CAPABILITY,
             require_extension: bool = True, deps: Deps | None = None) -> GpuSession:
    """Open this process's GPU after the checks of the module docstring; raises :class:`DeviceGuardError`."""
    global _ACTIVE
    deps = deps or Deps()
    env = deps.environ
    if _ACTIVE is not None:
        raise DeviceGuardError(f"a GPU session ({_ACTIVE.device}) is already open in this process")
    index = int(env.get("LOCAL_RANK", 0)) if local_index is None else int(local_index)
    if not deps.cuda_available():
        raise DeviceGuardError("no CUDA device is visible to this process")
    count = deps.device_count()
    if not 0 <= index < count:
        raise DeviceGuardError(f"device index {index} is out of range: {count} visible device(s)")
    cap = tuple(deps.capability(index))
    if require_capability is not None and cap != tuple(require_capability):
        raise DeviceGuardError(f"device {index} has compute capability {cap[0]}.{cap[1]}; the kernels are built for "
                               f"sm_{require_capability[0]}{require_capability[1]}a")
    physical = physical_index(index, env)
    gpu_lock = None
    if lock and not _held_by_launcher(physical, env):
        gpu_lock = GpuLock(lock_path(physical, lock_dir or default_lock_dir(env)))
        gpu_lock.acquire()
    try:
        free, total = deps.mem_get_info(index)
        if free < min_free_bytes:
            raise DeviceGuardError(f"device {index} has {free / 2**30:.1f} GiB free of {total / 2**30:.1f} GiB; "
                                   f"{min_free_bytes / 2**30:.1f} GiB required")
        if require_extension:
            try:
                deps.load_extension()
            except Exception as exc:
                raise DeviceGuardError(f"the kernel extension does not load: {exc}") from exc
        deps.set_device(index)
    except BaseException:
        if gpu_lock is not None:
            gpu_lock.release()
        raise
    session = GpuSession(index, physical, gpu_lock, deps)
    _ACTIVE = session
    atexit.register(session.close)
    return session


def acquire_gpu(local_index: int | None = None, **kwargs) -> GpuSession:
    """The open session if there is one (its owner keeps it), else a new one from :func:`open_gpu`. A request for a
    different device than the open one is refused."""
    if _ACTIVE is not None:
        want = _ACTIVE.index if local_index is None else int(local_index)
        if want != _ACTIVE.index:
            raise DeviceGuardError(f"{_ACTIVE.device} is open; cannot switch to cuda:{want} in the same process")
        return _ACTIVE
    return open_gpu(local_index, **kwargs)


def active_session() -> GpuSession | None:
    return _ACTIVE


__all__ = ["DeviceGuardError", "Deps", "GpuLock", "GpuSession", "LOCKS_HELD_ENV", "LOCK_DIR_ENV", "acquire_gpu",
           "active_session", "default_lock_dir", "lock_path", "open_gpu", "physical_index"]
