"""Host model of the two-shot gradient exchange of the fused Adam kernel (``adam_two_shot`` in
``ops/csrc/rl_kernels.cu``), with threads as ranks.

Per exchange ``e`` (epoch), with two send buffers per rank (alternating by parity), one reduced buffer per rank (the
averaged shard followed by the squared-norm slot) and one flag array per rank:

1. write this step's gradients into send buffer ``e % 2``; publish ``2 e`` (round 1) into every rank's flag array and
   wait until every slot of the own array holds at least ``2 e``;
2. average the own shard over all ranks in rank order into the reduced buffer, with its squared norm in the slot;
   publish ``2 e + 1`` (round 2) and wait for it from every rank;
3. sum the ranks' norm slots in rank order (the same global norm on every rank), clip, and apply Adam to the whole
   vector with each element's average read from the rank that owns its shard (parameters and moments replicated).

The model checks that two rounds make a single reduced buffer safe: a rank rewrites its reduced buffer only in step 2
of exchange ``e + 1``, after round 1 of ``e + 1``, which every rank publishes only once it has finished reading the
reduced buffers of exchange ``e``; that without round 2 a rank can read a shard its owner has not averaged yet; that
replicas are bit-identical every step; and that the result equals the one-shot exchange up to the summation order of
the norm. (The send buffers alternate by parity as the one-shot exchange needs; in the two-round protocol a rank reads
peers' send buffers only before it publishes round 2, so even one buffer would be safe there.)
"""

import threading
import time

import numpy as np
import pytest

P = 96  # parameters (the shards are ceil(P / W) long, the last one shorter)
LR, B1, B2, EPS, MAX_NORM = 1e-2, 0.9, 0.999, 1e-8, 0.5


def grads(rank: int, step: int) -> np.ndarray:
    g = np.random.default_rng(1000 * step + rank).standard_normal(P).astype(np.float32)
    return g * np.float32(0.2)


class Fabric:
    def __init__(self, world: int, send_buffers: int = 2) -> None:
        self.world = world
        self.nsend = send_buffers
        self.send = [[np.zeros(P, np.float32) for _ in range(send_buffers)] for _ in range(world)]
        self.reduced = [np.zeros(P + 1, np.float32) for _ in range(world)]  # shard values + norm slot at [P]
        self.flags = [[0] * world for _ in range(world)]  # flags[dst][src]
        self.lock = threading.Lock()
        self.violations = []

    def publish(self, rank: int, value: int) -> None:
        with self.lock:
            for r in range(self.world):
                self.flags[r][rank] = value

    def wait(self, rank: int, value: int, timeout_s: float = 10.0) -> None:
        t0 = time.monotonic()
        while True:
            with self.lock:
                if all(f >= value for f in self.flags[rank]):
                    return
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"rank {rank} waits for {value}")
            time.sleep(1e-4)


def shard_bounds(world: int, rank: int) -> tuple[int, int]:
    size = -(-P // world)
    return min(P, rank * size), min(P, (rank + 1) * size)


def owner(world: int, e: int) -> int:
    return e // -(-P // world)


def adam(p, g, m, v, step):
    m[:] = B1 * m + (1 - B1) * g
    v[:] = B2 * v + (1 - B2) * g * g
    bc1, bc2 = 1 - B1 ** step, 1 - B2 ** step
    p -= np.float32(LR / bc1) * m / (np.sqrt(v) / np.float32(np.sqrt(bc2)) + np.float32(EPS))


def two_shot_rank(fab: Fabric, rank: int, steps: int, out: dict, jitter, round2: bool = True) -> None:
    W = fab.world
    lo, hi = shard_bounds(W, rank)
    p = np.ones(P, np.float32)
    m, v = np.zeros(P, np.float32), np.zeros(P, np.float32)
    try:
        for step in range(steps):
            epoch = step + 1
            send = fab.send[rank][epoch % fab.nsend]
            send[:] = grads(rank, step)
            fab.publish(rank, 2 * epoch)
            fab.wait(rank, 2 * epoch)
            jitter()
            shard = np.zeros(hi - lo, np.float32)
            for r in range(W):  # rank order
                got = fab.send[r][epoch % fab.nsend][lo:hi].copy()
                if not np.array_equal(got, grads(r, step)[lo:hi]):
                    fab.violations.append(("send", rank, r, step))
                shard += got
                jitter()
            shard /= np.float32(W)
            fab.reduced[rank][lo:hi] = shard
            fab.reduced[rank][P] = np.float32(np.sum(shard * shard, dtype=np.float32))
            fab.publish(rank, 2 * epoch + 1)
            if round2:
                fab.wait(rank, 2 * epoch + 1)
            total = np.float32(0.0)
            for r in range(W):
                total += fab.reduced[r][P]
                jitter()
            coef = min(np.float32(MAX_NORM) / (np.sqrt(total) + np.float32(1e-6)), np.float32(1.0))
            g = np.empty(P, np.float32)
            for e in range(P):
                g[e] = fab.reduced[owner(W, e)][e]
            jitter()
            expect = np.mean(np.stack([grads(r, step) for r in range(W)]), axis=0)
            if not np.allclose(g, expect, rtol=1e-5, atol=1e-6):
                fab.violations.append(("reduced", rank, step))
            adam(p, g * coef, m, v, epoch)
            out.setdefault(rank, []).append(p.copy())
    except Exception as exc:  # reported to the test
        out[rank] = exc


def one_shot(world: int, steps: int) -> list[np.ndarray]:
    p = np.ones(P, np.float32)
    m, v = np.zeros(P, np.float32), np.zeros(P, np.float32)
    hist = []
    for step in range(steps):
        g = np.zeros(P, np.float32)
        for r in range(world):
            g += grads(r, step)
        g /= np.float32(world)
        norm = np.sqrt(np.sum(g * g, dtype=np.float32))
        coef = min(np.float32(MAX_NORM) / (norm + np.float32(1e-6)), np.float32(1.0))
        adam(p, g * coef, m, v, step + 1)
        hist.append(p.copy())
    return hist


def _run(world: int, steps: int, jitter, round2: bool = True):
    fab = Fabric(world)
    out = {}
    threads = [threading.Thread(target=two_shot_rank, args=(fab, r, steps, out, jitter(r), round2))
               for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    return fab, out


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_two_shot_protocol_is_race_free_and_replicas_match(world):
    rng = np.random.default_rng(world)
    lock = threading.Lock()

    def jitter(rank):
        def f():
            with lock:
                d = rng.uniform(0, 4e-4)
            time.sleep(d)
        return f

    steps = 12
    fab, out = _run(world, steps, jitter)
    errors = {r: v for r, v in out.items() if isinstance(v, Exception)}
    assert not errors and not fab.violations, (errors, fab.violations[:5])
    for step in range(steps):
        for r in range(1, world):
            assert np.array_equal(out[r][step], out[0][step])  # bit-identical replicas every step
    ref = one_shot(world, steps)
    for step in range(steps):
        np.testing.assert_allclose(out[0][step], ref[step], rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("round2,safe", [(True, True), (False, False)])
def test_round_two_is_what_makes_the_owners_shards_complete(round2, safe):
    """Rank 0 averages its shard slowly: without waiting for round 2, rank 1 reads rank 0's shard before it is
    written (stale values from the previous exchange)."""

    def jitter(rank):
        return (lambda: time.sleep(2e-3)) if rank == 0 else (lambda: None)

    fab, out = _run(2, 4, jitter, round2)
    assert (not fab.violations) == safe
