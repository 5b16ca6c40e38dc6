"""Host model of the gradient-exchange protocol of the fused Adam kernel (``ops/csrc/rl_kernels.cu:adam_step_kernel``),
with threads as ranks.

Per step a rank writes its gradients into send buffer ``epoch & 1`` (the kernels before the exchange), publishes
``epoch`` into its slot of every peer's flag array, waits until every peer's flag in its own array reached ``epoch``
(bounded), then reads every peer's buffer of that parity in rank order. The model checks what the kernel relies on:
with two buffers alternating by parity, a fast rank never overwrites gradients that a slow peer is still reading;
with one buffer it would. A rank that never publishes makes the others give up with a timeout instead of hanging.
"""

import threading
import time

import numpy as np
import pytest

N_ELEM = 64


class Exchange:
    def __init__(self, world: int, parity_buffers: int = 2, timeout_s: float = 5.0) -> None:
        self.world = world
        self.nbuf = parity_buffers
        self.send = [[np.zeros(N_ELEM) for _ in range(parity_buffers)] for _ in range(world)]
        self.flags = [[0] * world for _ in range(world)]  # flags[r][s]: epoch rank s published to rank r
        self.lock = threading.Lock()
        self.timeout_s = timeout_s

    def publish(self, rank: int, epoch: int) -> None:
        with self.lock:  # stands for st.release.sys after the gradient writes
            for r in range(self.world):
                self.flags[r][rank] = epoch

    def wait(self, rank: int, epoch: int) -> bool:
        t0 = time.monotonic()
        while True:
            with self.lock:  # ld.acquire.sys
                if all(f - epoch >= 0 for f in self.flags[rank]):
                    return True
            if time.monotonic() - t0 > self.timeout_s:
                return False  # the kernel records a timeout in its status word and leaves the parameters alone
            time.sleep(1e-4)


def grads(rank: int, step: int) -> np.ndarray:
    return np.full(N_ELEM, 1000.0 * step + rank)


def run_rank(ex: Exchange, rank: int, steps: int, out: dict, hooks=None) -> None:
    epoch = 0
    seen = []
    for step in range(steps):
        epoch += 1
        buf = ex.send[rank][epoch % ex.nbuf]
        buf[:] = grads(rank, step)  # gradient kernels of this step
        if hooks and "after_write" in hooks:
            hooks["after_write"](rank, step)
        ex.publish(rank, epoch)
        if not ex.wait(rank, epoch):
            out[rank] = ("timeout", step)
            return
        total = np.zeros(N_ELEM)
        for r in range(ex.world):  # rank order: identical sums on every rank
            if hooks and "before_read" in hooks:
                hooks["before_read"](rank, step, r)
            got = ex.send[r][epoch % ex.nbuf].copy()
            if not np.array_equal(got, grads(r, step)):
                out[rank] = ("stale", step, r, float(got[0]))
                return
            total += got
        seen.append(total / ex.world)
    out[rank] = ("ok", seen)


def _run(world, steps, nbuf, hooks=None, timeout_s=5.0, skip=None):
    ex = Exchange(world, nbuf, timeout_s)
    out = {}
    threads = [threading.Thread(target=run_rank, args=(ex, r, steps, out, hooks)) for r in range(world)
               if r != skip]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_parity_buffers_give_every_rank_the_same_average_under_random_delays(world):
    rng = np.random.default_rng(world)
    lock = threading.Lock()

    def jitter(*_):
        with lock:
            d = rng.uniform(0, 2e-3)
        time.sleep(d)

    out = _run(world, 25, 2, {"after_write": jitter, "before_read": jitter})
    assert all(v[0] == "ok" for v in out.values()), out
    ref = out[0][1]
    for r in range(world):
        for a, b in zip(out[r][1], ref):
            assert np.array_equal(a, b)  # bit-identical replicas
    for step, avg in enumerate(ref):
        assert np.allclose(avg, np.mean([grads(r, step) for r in range(world)], axis=0))


@pytest.mark.parametrize("nbuf,expect", [(1, "stale"), (2, "ok")])
def test_a_fast_rank_overwrites_a_slow_readers_data_only_with_one_buffer(nbuf, expect):
    """Rank 1 reads rank 0's step-0 gradients only after rank 0 has written its step-1 gradients."""
    wrote_next = threading.Event()

    def after_write(rank, step):
        if rank == 0 and step == 1:
            wrote_next.set()

    def before_read(rank, step, r):
        if rank == 1 and step == 0 and r == 0:
            assert wrote_next.wait(10)

    out = _run(2, 3, nbuf, {"after_write": after_write, "before_read": before_read}, timeout_s=1.0)
    assert out[1][0] == expect, out
    if expect == "ok":
        assert out[0][0] == "ok"


def test_a_rank_that_never_publishes_times_out_the_others():
    out = _run(3, 2, 2, timeout_s=0.3, skip=2)
    assert out[0] == ("timeout", 0) and out[1] == ("timeout", 0)
