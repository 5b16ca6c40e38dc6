"""Host model of a two-shot gradient exchange (reduce-scatter, Adam on a shard, all-gather of the parameters), with
threads as ranks: the protocol planned for the fused Adam kernel at 4-8 GPUs, where the one-shot exchange reads
(N - 1) full gradient vectors per rank and the two-shot moves 2 (N - 1) / N of one.

Per step, with one send buffer, one norm slot and one parameter buffer per rank:

1. write this step's gradients into the send buffer, publish flag 1, wait for flag 1 of every rank;
2. sum the own shard over all ranks in rank order, divide by N; square-sum per clip group into the own norm slot;
   publish flag 2, wait for flag 2 of every rank;
3. read every rank's norm slot in rank order (the same global norms on every rank), clip, adaptive learning rate,
   Adam on the own shard (moments are sharded);
4. store the updated shard into every rank's parameter buffer, publish flag 3, wait for flag 3 of every rank.

The model checks that the three flag rounds make one buffer of each kind safe (no rank overwrites data a peer still
reads), that every rank ends each step with bit-identical parameters, and that they equal the one-shot result up to
the summation order of the norms.
"""

import threading
import time

import numpy as np
import pytest

P = 96  # parameters (divisible by every world size tested)
LR, B1, B2, EPS, MAX_NORM = 1e-2, 0.9, 0.999, 1e-8, 0.5


def grads(rank: int, step: int) -> np.ndarray:
    g = np.random.default_rng(1000 * step + rank).standard_normal(P).astype(np.float32)
    return g * np.float32(0.2)


class Fabric:
    def __init__(self, world: int) -> None:
        self.world = world
        self.send = [np.zeros(P, np.float32) for _ in range(world)]
        self.norm = [np.zeros(1, np.float32) for _ in range(world)]
        self.params = [np.ones(P, np.float32) for _ in range(world)]
        self.flags = [[[0] * world for _ in range(world)] for _ in range(3)]  # flags[k][dst][src]
        self.lock = threading.Lock()
        self.violations = []

    def publish(self, k: int, rank: int, epoch: int) -> None:
        with self.lock:
            for r in range(self.world):
                self.flags[k][r][rank] = epoch

    def wait(self, k: int, rank: int, epoch: int, timeout_s: float = 10.0) -> None:
        t0 = time.monotonic()
        while True:
            with self.lock:
                if all(f >= epoch for f in self.flags[k][rank]):
                    return
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"rank {rank} flag {k + 1} epoch {epoch}")
            time.sleep(1e-4)


def adam(p, g, m, v, step):
    m[:] = B1 * m + (1 - B1) * g
    v[:] = B2 * v + (1 - B2) * g * g
    bc1, bc2 = 1 - B1 ** step, 1 - B2 ** step
    p -= np.float32(LR / bc1) * m / (np.sqrt(v) / np.float32(np.sqrt(bc2)) + np.float32(EPS))


def two_shot_rank(fab: Fabric, rank: int, steps: int, out: dict, jitter, rounds: int = 3, before_store=None) -> None:
    W = fab.world
    lo, hi = rank * P // W, (rank + 1) * P // W
    m, v = np.zeros(hi - lo, np.float32), np.zeros(hi - lo, np.float32)
    try:
        for step in range(steps):
            epoch = step + 1
            fab.send[rank][:] = grads(rank, step)
            fab.publish(0, rank, epoch)
            fab.wait(0, rank, epoch)
            jitter()
            shard = np.zeros(hi - lo, np.float32)
            for r in range(W):
                got = fab.send[r][lo:hi].copy()
                if not np.array_equal(got, grads(r, step)[lo:hi]):
                    fab.violations.append(("send", rank, r, step))
                shard += got
                jitter()
            shard /= np.float32(W)
            fab.norm[rank][0] = np.float32(np.sum(shard * shard, dtype=np.float32))
            fab.publish(1, rank, epoch)
            fab.wait(1, rank, epoch)
            total = np.float32(0.0)
            for r in range(W):
                total += fab.norm[r][0]
                jitter()
            coef = min(np.float32(MAX_NORM) / (np.sqrt(total) + np.float32(1e-6)), np.float32(1.0))
            p = fab.params[rank][lo:hi].copy()
            adam(p, shard * coef, m, v, epoch)
            if before_store is not None:
                before_store(rank, step)
            for r in range(W):
                fab.params[r][lo:hi] = p
                jitter()
            if rounds == 3:
                fab.publish(2, rank, epoch)
                fab.wait(2, rank, epoch)
            out.setdefault(rank, []).append(fab.params[rank].copy())
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


@pytest.mark.parametrize("world", [2, 4, 8])
def test_two_shot_protocol_is_race_free_and_replicas_match(world):
    fab = Fabric(world)
    rng = np.random.default_rng(world)
    lock = threading.Lock()

    def jitter():
        with lock:
            d = rng.uniform(0, 4e-4)
        time.sleep(d)

    out, steps = {}, 12
    threads = [threading.Thread(target=two_shot_rank, args=(fab, r, steps, out, jitter)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    errors = {r: v for r, v in out.items() if isinstance(v, Exception)}
    assert not errors and not fab.violations, (errors, fab.violations[:5])
    for step in range(steps):
        for r in range(1, world):
            assert np.array_equal(out[r][step], out[0][step])  # bit-identical replicas every step
    ref = one_shot(world, steps)
    for step in range(steps):
        np.testing.assert_allclose(out[0][step], ref[step], rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("rounds,identical", [(3, True), (2, False)])
def test_the_third_flag_round_is_what_keeps_parameters_complete(rounds, identical):
    """Rank 0 is slow to store its updated shard: without the third flag round rank 1 goes on with stale
    parameters."""
    fab = Fabric(2)
    out = {}

    def slow_store(rank, step):
        if rank == 0 and step == 0:
            time.sleep(0.05)

    threads = [threading.Thread(target=two_shot_rank, args=(fab, r, 1, out, lambda: None, rounds, slow_store))
               for r in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    assert np.array_equal(out[0][0], out[1][0]) == identical
