"""Bounded device-side waits: a peer flag that nothing sets makes the kernel give up, record the failing site in the
status word and leave the parameters untouched. Both "ranks" live on one GPU; nothing faults, traps or hangs."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_adam_exchange_times_out_on_missing_peer():
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    dev = "cuda"
    n = 1000
    flat = torch.randn(n, device=dev)
    before = flat.clone()
    send = torch.randn(n + 4, device=dev)
    grads = torch.zeros(n + 4, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    tens, chunks, nch = C.make_adam_plan([0, n], [n, 4], [0, -1], [1, 1], [n, 4], [None, None], [0, 0], flat)
    grid = C.adam_grid(torch.cuda.current_device())
    flags0 = torch.zeros(2, dtype=torch.int32, device=dev)  # rank 0's flag array: slot 1 is never written
    flags1 = torch.zeros(2, dtype=torch.int32, device=dev)  # "rank 1" array (receives rank 0's publication)
    peer_send = torch.tensor([send.data_ptr()] * 4, dtype=torch.int64, device=dev)
    peer_flags = torch.tensor([flags0.data_ptr(), flags1.data_ptr()], dtype=torch.int64, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    lr = torch.tensor([1e-3], device=dev)
    step = torch.zeros(1, dtype=torch.int64, device=dev)
    C.adam_step(flat, send, send, grads, m, v, tens, chunks, nch, [1.0], [0.9], [0.999], [1e-8], [0], lr, None, step,
                False, None, 0.01, 1e-5, 1e-2, 2, 0, peer_send, peer_flags, epoch, 200 * 10**6,
                torch.zeros(grid * 4, device=dev), torch.zeros(4, dtype=torch.int32, device=dev), status, None, grid,
                [0, n], n + 4)
    torch.cuda.synchronize()
    st = status.tolist()
    assert st[0] == 4  # peer-flag timeout
    assert torch.equal(flat, before)
    assert int(flags1[0]) == 1  # rank 0 did publish its epoch to the peer
    # the context is still usable
    assert float((flat * 2).sum()) == pytest.approx(float(before.sum() * 2), rel=1e-5)


def test_small_collective_times_out_on_missing_peer():
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    dev = "cuda"
    buf0 = torch.randn(16, dtype=torch.float64, device=dev)
    buf1 = torch.randn(16, dtype=torch.float64, device=dev)
    flags0 = torch.zeros(2, dtype=torch.int32, device=dev)
    flags1 = torch.zeros(2, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    out = torch.full((16,), -1.0, dtype=torch.float64, device=dev)
    C.p2p_allreduce_f64([buf0.data_ptr(), buf1.data_ptr()], [flags0.data_ptr(), flags1.data_ptr()], 0, epoch,
                        100 * 10**6, status, out, 16)
    torch.cuda.synchronize()
    assert status[0].item() == 4
    assert torch.all(out == -1.0)


def test_small_collective_completes_when_peer_flag_is_set():
    """Same single-GPU emulation, with the missing peer's flags set in advance: the sum is rank ordered."""
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    dev = "cuda"
    buf0 = torch.randn(16, dtype=torch.float64, device=dev)
    buf1 = torch.randn(16, dtype=torch.float64, device=dev)
    flags0 = torch.tensor([0, 2], dtype=torch.int32, device=dev)  # "rank 1" already published epochs 1 and 2
    flags1 = torch.zeros(2, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    out = torch.zeros(16, dtype=torch.float64, device=dev)
    C.p2p_allreduce_f64([buf0.data_ptr(), buf1.data_ptr()], [flags0.data_ptr(), flags1.data_ptr()], 0, epoch,
                        10**9, status, out, 16)
    torch.cuda.synchronize()
    assert status[0].item() == 0
    assert torch.equal(out, buf0 + buf1)
    assert int(epoch) == 2
