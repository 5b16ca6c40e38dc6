"""The allocation-free C entry point ``rlb_gae_advantages_noalloc`` (declared in ``ops/csrc/gae_noalloc.h``).

The entry point exists for callers that may not allocate device memory while running (a C/C++ learner inside a
fixed-memory control process, or host code without PyTorch's caching allocator): its scratch space is a fixed device
array inside the library. This test calls it through its exported C symbol, with the argument types read from the
header, twice in a row on different data (odd N), and compares each result bit for bit with the regular entry point
(the same kernels with a caller-allocated scratch buffer) and with a plain PyTorch fp32 GAE + unbiased-std
normalisation; a call without normalisation must return advantages equal to returns - values exactly.
This file is collected last so that a run stopping at the first failure has already run every other test.
"""

import ctypes
import pathlib
import re

import pytest
import torch

pytestmark = pytest.mark.gpu

HEADER = pathlib.Path(__file__).resolve().parents[1] / "tt_rsl_rl_b200" / "ops" / "csrc" / "gae_noalloc.h"
_CTYPES = {"const float*": ctypes.c_void_p, "float*": ctypes.c_void_p, "int": ctypes.c_int, "float": ctypes.c_float,
           "cudaStream_t": ctypes.c_void_p}


def header_signature() -> list[str]:
    """Parameter types of the declaration in the header."""
    decl = re.search(r"int\s+rlb_gae_advantages_noalloc\s*\(([^)]*)\)", HEADER.read_text()).group(1)
    return [" ".join(p.split()[:-1]).replace(" *", "*") for p in decl.split(",")]


def max_envs() -> int:
    """RLB_GAE_NOALLOC_MAX_ENVS of the header, written as ``(a << b)``."""
    a, b = re.search(r"#define RLB_GAE_NOALLOC_MAX_ENVS \((\d+) << (\d+)\)", HEADER.read_text()).groups()
    return int(a) << int(b)


def _lib():
    import tt_rsl_rl_b200._C as C  # noqa: F401 - loads the shared library into the process

    lib = ctypes.CDLL(C.__file__)
    fn = lib.rlb_gae_advantages_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [_CTYPES[t] for t in header_signature()]
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


def _torch_gae(rewards, dones, values, last, T, N, gamma, lam):
    """fp32 PyTorch definition (``rsl_rl/algorithms/ppo.py:166-191``): GAE, then (A - mean) / (unbiased std + 1e-8)."""
    r, d, v = rewards.view(T, N), dones.view(T, N), values.view(T, N)
    ret = torch.empty_like(r)
    adv = torch.zeros(N, device=r.device)
    for t in range(T - 1, -1, -1):
        nxt = last if t == T - 1 else v[t + 1]
        alive = 1.0 - d[t]
        delta = r[t] + alive * gamma * nxt - v[t]
        adv = delta + alive * gamma * lam * adv
        ret[t] = adv + v[t]
    a = (ret - v).reshape(-1)
    return ret.reshape(-1), (a - a.mean()) / (a.std() + 1e-8)


def test_noalloc_entry_point_matches_regular_entry_point_and_torch():
    fn = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    gamma, lam = 0.99, 0.95
    for call, (T, N) in enumerate([(24, 5001), (16, 70001)]):  # two calls in a row, odd N
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
        # the same kernels in the same order: bit for bit
        torch.testing.assert_close(ret, ret_ref, atol=0, rtol=0)
        torch.testing.assert_close(adv, adv_ref, atol=0, rtol=0)
        ret_t, adv_t = _torch_gae(rewards, dones, values, last, T, N, gamma, lam)
        torch.testing.assert_close(ret, ret_t, atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(adv, adv_t, atol=1e-5, rtol=1e-4)
        # without normalisation: advantages = returns - values, exactly
        adv_raw = torch.full((T * N,), float("nan"), device="cuda")
        rc = fn(rewards.data_ptr(), dones.data_ptr(), values.data_ptr(), last.data_ptr(), ret.data_ptr(),
                adv_raw.data_ptr(), T, N, gamma, lam, 0, stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(adv_raw, ret - values)


def test_noalloc_entry_point_rejects_oversized_batches():
    fn = _lib()
    t = torch.zeros(8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, max_envs() + 1,
            0.99, 0.95, 1, stream)
    assert rc == 1  # cudaErrorInvalidValue, nothing launched
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 0, 8, 0.99, 0.95, 1,
            stream)
    assert rc == 1
