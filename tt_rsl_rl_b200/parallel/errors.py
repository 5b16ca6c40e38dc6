"""Errors raised by the communicator and the device status word. The replica check mirrors the reference plugin's
(``rsl_rl_tt/ppo.py:678-698``); upstream rsl_rl raises neither."""


class CommTimeoutError(RuntimeError):
    """A device-side wait ran out (peer flag, grid barrier or pipeline stage) or a rank failed to join in time.

    The kernels record the first failing site in a status word and return instead of hanging; the host reads the word
    after each update and raises this error.
    """


class ReplicaDivergenceError(RuntimeError):
    """Data-parallel replicas no longer hold identical parameters (raised on every rank by the replica check)."""
