"""The allocation-free C entry point ``rlb_gae_advantages_noalloc`` against the regular GAE entry point.

The entry point exists for callers that may not allocate device memory while running (a C/C++ learner inside a
fixed-memory control process, or host code without PyTorch's caching allocator): its scratch space is a fixed device
array inside the library. This test calls it through its exported C symbol, twice in a row on different data, and
compares each result with the regular entry point (which takes a caller-allocated scratch buffer).
This file is collected last so that a run stopping at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ENVS = 1 << 20


def _lib():
    import tt_rsl_rl_b200._C as C  # noqa: F401 - loads the shared library into the process

    lib = ctypes.CDLL(C.__file__)
    fn = lib.rlb_gae_advantages_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                           ctypes.c_void_p]
    return fn


def _regular(rewards, dones, values, last, T, N, gamma, lam):
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    ret = torch.empty(T * N, device="cuda")
    adv = torch.empty(T * N, device="cuda")
    partial = torch.empty(2 * C.gae_blocks(N), dtype=torch.float64, device="cuda")
    C.gae(rewards, dones, values, last, ret, adv, T, N, gamma, lam, partial)
    C.adv_normalize(adv, partial, C.gae_blocks(N))
    return ret, adv


def test_noalloc_entry_point_matches_regular_entry_point():
    fn = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    gamma, lam = 0.99, 0.95
    for call, (T, N) in enumerate([(24, 5000), (16, 70001)]):
        g = torch.Generator(device="cuda").manual_seed(call)
        rewards = torch.randn(T * N, device="cuda", generator=g)
        dones = (torch.rand(T * N, device="cuda", generator=g) < 0.05).float()
        values = torch.randn(T * N, device="cuda", generator=g)
        last = torch.randn(N, device="cuda", generator=g)
        ret_ref, adv_ref = _regular(rewards, dones, values, last, T, N, gamma, lam)
        ret = torch.full((T * N,), float("nan"), device="cuda")
        adv = torch.full((T * N,), float("nan"), device="cuda")
        rc = fn(rewards.data_ptr(), dones.data_ptr(), values.data_ptr(), last.data_ptr(), ret.data_ptr(),
                adv.data_ptr(), T, N, gamma, lam, 1, stream)
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(ret, ret_ref, atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(adv, adv_ref, atol=1e-5, rtol=1e-4)


def test_noalloc_entry_point_rejects_oversized_batches():
    fn = _lib()
    t = torch.zeros(8, device="cuda")
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, MAX_ENVS + 1, 0.99,
            0.95, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # cudaErrorInvalidValue, nothing launched
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 0, 8, 0.99, 0.95, 1,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
