"""Symmetric device buffers shared by the ranks of one node, and the collectives built on them.

One process per GPU (``torchrun``). ``torch.distributed`` is used once, at construction, to exchange CUDA IPC handles
(``all_gather_object``); afterwards every exchange is a kernel reading peer memory over NVLink / NVSwitch:

* gradient exchange: two send buffers per rank (alternating by exchange parity, so a rank never overwrites gradients a
  slower peer may still read), a reduced buffer (the rank's averaged shard and its squared norms, for the two-shot
  exchange) and a flag array; consumed by the fused clip + Adam kernel, which sums the ranks' gradients in rank order
  (every element on every rank in the one-shot exchange, the own shard in the two-shot one), so every rank computes
  bit-identical parameters;
* small collectives (normaliser moments, parameter broadcast) on a separate buffer and flag channel.

Replaces ``torch.distributed`` all-reduce / broadcast at ``rsl_rl/utils/utils.py:345-392``,
``rsl_rl/algorithms/ppo.py:248,261,467-486`` and ``rsl_rl/modules/normalization.py:62-71``.
Every device wait is bounded (``timeout_ms``); a timeout sets the engine's status word and the host raises
:class:`CommTimeoutError`.
"""

from __future__ import annotations

import torch

from ..ops import ext


class PeerExchange:
    def __init__(self, n_exchange: int, n_small_bytes: int, rank: int, world: int, device: torch.device,
                 timeout_ms: float = 10000.0) -> None:
        if world > 8:
            raise ValueError("the peer exchange supports up to 8 ranks (one node)")
        C = ext()
        self.rank = rank
        self.world = world
        self.device = device
        self.timeout_ns = int(timeout_ms * 1e6)
        dev = device.index
        self._bufs = {
            "send0": C.ipc_alloc(4 * n_exchange, dev),
            "send1": C.ipc_alloc(4 * n_exchange, dev),
            "reduced": C.ipc_alloc(4 * (n_exchange + 8), dev),
            "flags": C.ipc_alloc(4 * world, dev),
            "small": C.ipc_alloc(max(64, n_small_bytes), dev),
            "small_flags": C.ipc_alloc(4 * world, dev),
        }
        self.send = [self._bufs["send0"].view(torch.float32), self._bufs["send1"].view(torch.float32)]
        self.small = self._bufs["small"]
        self.small_epoch = torch.zeros(1, dtype=torch.int32, device=device)
        handles = {k: C.ipc_handle(v) for k, v in self._bufs.items()}
        gathered: list = [None] * world
        torch.distributed.all_gather_object(gathered, handles)
        self._opened: list[int] = []
        ptrs: dict[str, list[int]] = {k: [] for k in self._bufs}
        for r in range(world):
            for k in self._bufs:
                if r == rank:
                    ptrs[k].append(self._bufs[k].data_ptr())
                else:
                    p = C.ipc_open(gathered[r][k], dev)
                    self._opened.append(p)
                    ptrs[k].append(p)
        self.ptrs = ptrs
        # device pointer tables read by the fused Adam kernel
        self.peer_send = torch.tensor(ptrs["send0"] + ptrs["send1"], dtype=torch.int64, device=device)
        self.peer_flags = torch.tensor(ptrs["flags"], dtype=torch.int64, device=device)
        self.peer_reduced = torch.tensor(ptrs["reduced"], dtype=torch.int64, device=device)
        torch.distributed.barrier()

    @classmethod
    def create(cls, n_exchange: int, n_small_bytes: int, rank: int, world: int, device: torch.device,
               timeout_ms: float = 10000.0) -> PeerExchange:
        return cls(n_exchange, n_small_bytes, rank, world, device, timeout_ms)

    # ---- small collectives ------------------------------------------------------------------------------------------
    def allreduce_f64(self, local: torch.Tensor, out: torch.Tensor, status: torch.Tensor | None = None) -> None:
        """``out = sum over ranks of local`` (float64, rank-ordered, identical on every rank)."""
        n = local.numel()
        if n * 8 > self.small.numel():
            raise ValueError("allreduce_f64: buffer too small")
        self.small[: n * 8].view(torch.float64).copy_(local.reshape(-1))
        ext().p2p_allreduce_f64(self.ptrs["small"], self.ptrs["small_flags"], self.rank, self.small_epoch,
                                self.timeout_ns, status, out, n)

    def broadcast_(self, t: torch.Tensor, root: int = 0, status: torch.Tensor | None = None) -> None:
        """Overwrite ``t`` on every rank with rank ``root``'s values (bitwise; any dtype of 4-byte multiples)."""
        nbytes = t.numel() * t.element_size()
        if nbytes % 4 or nbytes > self.small.numel():
            raise ValueError("broadcast_: unsupported size")
        if not t.is_contiguous():
            raise ValueError("broadcast_: tensor must be contiguous")
        raw = t.reshape(-1).view(torch.uint8)
        words = raw.view(torch.float32)
        if self.rank == root:
            self.small[:nbytes].copy_(raw)
        ext().p2p_broadcast_f32(self.ptrs["small"], self.ptrs["small_flags"], self.rank, self.small_epoch,
                                self.timeout_ns, status, root, words, nbytes // 4)

    def close(self) -> None:
        C = ext()
        for p in self._opened:
            C.ipc_close(p)
        self._opened.clear()

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass
