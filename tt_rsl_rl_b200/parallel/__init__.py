"""Data-parallel communication: the peer-to-peer gradient exchange used inside the fused Adam kernel, parameter
broadcast and normaliser-statistics combine, with bounded device-side waits and host-side failure reporting."""

from .errors import CommTimeoutError, ReplicaDivergenceError
from .replica import ReplicaChecker

__all__ = ["CommTimeoutError", "PeerExchange", "ReplicaChecker", "ReplicaDivergenceError"]


def __getattr__(name):
    if name == "PeerExchange":
        from .peer_exchange import PeerExchange

        return PeerExchange
    raise AttributeError(name)
