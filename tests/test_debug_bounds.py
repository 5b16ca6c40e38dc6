"""Bounds-checked debug builds: the status code a bad index reports, its host-side error, and the build switch.

Kernels that read indices from memory check them with ``RL_CHECK_INDEX`` when built with ``-DRL_DEBUG_BOUNDS``; an
index outside its tensor is recorded in the status word and replaced by 0. The GPU side is a compile-time switch, so
these host tests check the mapping of the status word and that release builds define the check away.
"""

from __future__ import annotations

import os
import re
import types

import pytest
import torch

from tt_rsl_rl_b200.engine.base import EngineBase
from tt_rsl_rl_b200.parallel import CommTimeoutError

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PRIMS = os.path.join(ROOT, "tt_rsl_rl_b200", "ops", "csrc", "sm100_primitives.cuh")


def _engine_with_status(words):
    eng = types.SimpleNamespace(status=torch.tensor(words, dtype=torch.int64))
    return eng


def test_bad_index_status_raises_index_error_and_clears_the_word():
    eng = _engine_with_status([8, 41, 3, 2])
    with pytest.raises(IndexError, match="site=41 block=3 count=2"):
        EngineBase._check_status(eng)
    assert int(eng.status.abs().sum()) == 0


def test_timeouts_still_raise_comm_timeout():
    eng = _engine_with_status([4, 60, 0, 1])
    with pytest.raises(CommTimeoutError):
        EngineBase._check_status(eng)
    EngineBase._check_status(_engine_with_status([0, 0, 0, 0]))  # a clean word raises nothing


def test_status_code_of_bad_index_matches_the_host_mapping():
    src = open(PRIMS).read()
    assert re.search(r"kBadIndex\s*=\s*8\b", src)
    # the release branch of the macro is empty: default builds carry no check
    release = src.split("#else", 1)[1].split("#endif", 1)[0]
    assert "RL_CHECK_INDEX" in release and "report_error" not in release


def test_setup_adds_the_define_only_when_asked(monkeypatch):
    text = open(os.path.join(ROOT, "setup.py")).read()
    assert 'os.environ.get("TT_RSL_RL_DEBUG_BOUNDS") == "1"' in text and "-DRL_DEBUG_BOUNDS" in text


def test_loaded_build_reports_its_bounds_mode():
    """The extension says which build is loaded (release builds: no checks), so logs and tests can record it."""
    from tt_rsl_rl_b200.ops import ext

    assert ext().debug_bounds_enabled() is (os.environ.get("TT_RSL_RL_DEBUG_BOUNDS") == "1")


def test_every_index_read_from_memory_has_a_check_site():
    """Sites: 41 minibatch gather sample index, 42 mirrored copy source column, 43 per-minibatch advantage index,
    44 loss kernels' storage row, 45 mirrored action column."""
    src = open(os.path.join(ROOT, "tt_rsl_rl_b200", "ops", "csrc", "rl_kernels.cu")).read()
    sites = sorted(int(s) for s in re.findall(r"RL_CHECK_INDEX\([^;]*,\s*(\d+)\);", src))
    assert sorted(set(sites)) == [41, 42, 43, 44, 45]


@pytest.mark.gpu
def test_debug_build_reports_a_bad_gather_index():
    """Debug builds only: a sample index past the rollout is reported as site 41 and read as row 0. The storage
    is allocated larger than the rollout, so the index stays inside the allocation even without the check."""
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    if not C.debug_bounds_enabled():
        pytest.skip("release build: no index checks (build with TT_RSL_RL_DEBUG_BOUNDS=1)")
    total, B, D = 64, 32, 8
    obs = torch.randn(total + 16, D, device="cuda")
    idx_in = torch.arange(B, dtype=torch.int32, device="cuda")
    idx_in[5] = total + 3
    idx_out = torch.zeros(B, dtype=torch.int32, device="cuda")
    x = torch.zeros(B, D, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    C.gather_minibatch(B, 0, total, None, 0, idx_in, idx_out, [obs], [None], [None], 0.0, [x], [D], status, 1, [B],
                       [None], [None])
    torch.cuda.synchronize()
    st = status.tolist()
    assert st[0] == 8 and st[1] == 41 and st[3] >= 1, st
    torch.testing.assert_close(x[5].float(), obs[0].bfloat16().float())
    good = [i for i in range(B) if i != 5]
    torch.testing.assert_close(x[good].float(), obs[good].bfloat16().float())
