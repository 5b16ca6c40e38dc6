"""Bounded device-side waits: a peer flag that nothing sets makes the kernel give up, record the failing site in the
status word and leave the parameters untouched. Both "ranks" live on one GPU; nothing faults, traps or hangs. The
two-shot exchange is also run to completion on one GPU, with the second rank's part (its flags and its averaged
shard) prepared by the test, and compared with the PyTorch definition of the step."""

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
                [0, n], n + 4, None, -1)
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


def _two_shot_setup(n=1000, seed=0):
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(seed)
    n_ex = (n + 4 + 3) // 4 * 4
    s0 = torch.randn(n_ex, device=dev, generator=g) * 0.1  # rank 0's gradients (this process)
    s1 = torch.randn(n_ex, device=dev, generator=g) * 0.1  # "rank 1"'s gradients
    red0 = torch.zeros(n_ex + 8, device=dev)
    red1 = torch.zeros(n_ex + 8, device=dev)
    flat = torch.randn(n, device=dev, generator=g)
    tens, chunks, nch = C.make_adam_plan([0, n], [n, 4], [0, -1], [1, 1], [n, 4], [None, None], [0, 0], flat)
    grid = C.adam_grid(torch.cuda.current_device())
    return C, dev, n, n_ex, s0, s1, red0, red1, flat, tens, chunks, nch, grid


def _two_shot_call(C, dev, n, n_ex, s0, s1, red0, red1, flat, tens, chunks, nch, grid, flags0, flags1, timeout_ns,
                   max_norm=0.5):
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    grads = torch.zeros(n_ex, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    lr = torch.tensor([1e-3], device=dev)
    step = torch.zeros(1, dtype=torch.int64, device=dev)
    # parity (epoch 1) & 1 = 1 selects the second half of the send table: [s0, s1]
    peer_send = torch.tensor([s0.data_ptr(), s1.data_ptr()] * 2, dtype=torch.int64, device=dev)
    peer_flags = torch.tensor([flags0.data_ptr(), flags1.data_ptr()], dtype=torch.int64, device=dev)
    peer_reduced = torch.tensor([red0.data_ptr(), red1.data_ptr()], dtype=torch.int64, device=dev)
    C.adam_step(flat, s0, s0, grads, m, v, tens, chunks, nch, [max_norm], [0.9], [0.999], [1e-8], [0], lr, None, step,
                False, None, 0.01, 1e-5, 1e-2, 2, 0, peer_send, peer_flags, epoch, timeout_ns,
                torch.zeros(grid * 4, device=dev), torch.zeros(4, dtype=torch.int32, device=dev), status, None, grid,
                [0, n], n_ex, peer_reduced, -1)
    torch.cuda.synchronize()
    return status, grads, m, v, epoch


def test_two_shot_exchange_times_out_on_missing_peer():
    C, dev, n, n_ex, s0, s1, red0, red1, flat, tens, chunks, nch, grid = _two_shot_setup()
    before = flat.clone()
    flags0 = torch.zeros(2, dtype=torch.int32, device=dev)  # slot 1 ("rank 1") never written
    flags1 = torch.zeros(2, dtype=torch.int32, device=dev)
    status, *_ = _two_shot_call(C, dev, n, n_ex, s0, s1, red0, red1, flat, tens, chunks, nch, grid, flags0, flags1,
                                200 * 10**6)
    assert status[0].item() == 4 and status[1].item() == 61  # round 1, waiting for rank 1
    assert torch.equal(flat, before)
    assert int(flags1[0]) == 2  # round 1 of exchange 1 was published to the peer


def test_two_shot_exchange_matches_the_torch_step():
    """Rank 0 of a two-rank two-shot exchange on one GPU: rank 1's flags (2 e, 2 e + 1) and its averaged shard with
    its squared-norm slot are prepared as rank 1 would have written them."""
    C, dev, n, n_ex, s0, s1, red0, red1, flat, tens, chunks, nch, grid = _two_shot_setup()
    before = flat.clone()
    avg = (s0 + s1) * 0.5  # rank-ordered sum, then the 1 / world factor: the kernel's arithmetic
    n4 = n_ex // 4
    shard = (n4 + 1) // 2 * 4  # elements of rank 0's shard
    red1[shard:n_ex] = avg[shard:]
    red1[n_ex] = avg[shard:n].square().sum()  # rank 1's group-0 squared norm (parameters only)
    flags0 = torch.tensor([0, 3], dtype=torch.int32, device=dev)  # rank 1 passed rounds 1 and 2 of exchange 1
    flags1 = torch.zeros(2, dtype=torch.int32, device=dev)
    status, grads, m, v, epoch = _two_shot_call(C, dev, n, n_ex, s0, s1, red0, red1, flat, tens, chunks, nch, grid,
                                                flags0, flags1, 10**9)
    assert status.tolist() == [0, 0, 0, 0]
    assert int(epoch) == 1 and int(flags1[0]) == 3  # both rounds published to the peer
    assert torch.equal(red0[:shard], avg[:shard])  # the own shard, averaged in rank order
    torch.testing.assert_close(red0[n_ex], avg[:min(shard, n)].square().sum(), rtol=1e-5, atol=1e-7)
    assert torch.equal(grads[:n_ex], avg)  # every element's average, read from its owner
    # the PyTorch definition: clip the averaged gradient to norm 0.5, one Adam step
    p = torch.nn.Parameter(before.clone())
    p.grad = avg[:n].clone()
    torch.nn.utils.clip_grad_norm_([p], 0.5)
    opt = torch.optim.Adam([p], lr=1e-3)
    opt.step()
    torch.testing.assert_close(flat, p.detach(), rtol=1e-6, atol=1e-7)
