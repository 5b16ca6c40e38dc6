"""Invariants of the source tree, checked on the host: no traps or device asserts, no batched-copy calls, no
compatibility layers, build notes not named from code, every kernel wait bounded."""

import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "tt_rsl_rl_b200"
CSRC = PKG / "ops" / "csrc"
CODE_EXT = {".py", ".cu", ".cuh", ".cpp", ".h", ".c"}


def _code_files():
    roots = [PKG, ROOT / "tests", ROOT / "baseline" / "compat"]
    files = [p for r in roots for p in r.rglob("*") if p.suffix in CODE_EXT and "__pycache__" not in p.parts]
    files += [ROOT / n for n in ("bench.py", "__graft_entry__.py", "setup.py") if (ROOT / n).exists()]
    return files


def _offenders(pattern, files):
    rx = re.compile(pattern)
    return [f"{p.relative_to(ROOT)}:{i}" for p in files for i, line in enumerate(p.read_text(errors="replace").splitlines(), 1)
            if rx.search(line)]


def test_no_traps_or_device_asserts():
    kernels = [p for p in CSRC.rglob("*") if p.suffix in {".cu", ".cuh"}]
    assert kernels
    assert _offenders(r"\b__" + "trap" + r"\b|asm[^;]*\btrap\b", kernels) == []
    assert _offenders(r"(?<![_\w])assert\s*\(", kernels) == []  # static_assert is fine


def test_no_batched_copy_calls():
    assert _offenders(r"[Cc]u(da)?Memcpy(3D)?" + "Batch", _code_files()) == []


def test_no_compatibility_layers_on_the_compute_path():
    pkg = [p for p in PKG.rglob("*.py")]
    assert _offenders(r"^\s*(import|from)\s+(triton|tilelang)\b", pkg) == []
    # torch.compile only behind the user's opt-in wrapper
    assert _offenders(r"torch\.compile\(", pkg) == ["tt_rsl_rl_b200/utils/utils.py:" + str(
        next(i for i, line in enumerate((PKG / "utils" / "utils.py").read_text().splitlines(), 1)
             if "torch.compile(" in line))]


def test_code_names_no_build_notes():
    notes = [p.stem for p in ROOT.glob("*.md") if p.name != "README.md"]
    assert notes
    pattern = r"\b(" + "|".join(re.escape(n) for n in notes) + r")(\.md)?\b"
    assert _offenders(pattern, _code_files()) == []


def test_every_kernel_wait_loop_is_bounded():
    """Each loop that polls memory written by another thread, block or GPU (acquire loads, mbarrier try-waits, a
    barrier generation) also reads the global timer and gives up after a deadline."""
    polling = re.compile(r"ld_acquire|try_wait|\*gen\b|volatile")
    bounded = re.compile(r"globaltimer|timeout")
    found = 0
    for p in CSRC.rglob("*"):
        if p.suffix not in {".cu", ".cuh"}:
            continue
        lines = p.read_text().splitlines()
        for i, line in enumerate(lines):
            if not re.search(r"\bwhile\s*\(|\bfor\s*\(\s*;\s*;", line):
                continue
            window = "\n".join(lines[i: i + 12])
            if polling.search(window):
                found += 1
                assert bounded.search(window), f"unbounded wait at {p.relative_to(ROOT)}:{i + 1}"
    assert found >= 4  # the peer-flag waits, the grid barrier and the mbarrier wait


def test_engines_read_device_data_only_through_named_transfers():
    """Every device-to-host read of the fused engines goes through ``HostTransfers.read`` with a tag, so the
    benchmark's count of reads per iteration is complete."""
    files = [p for p in (PKG / "engine").glob("*.py")] + [PKG / "parallel" / "peer_exchange.py"]
    assert _offenders(r"\.(item|tolist|cpu|numpy)\(\)", files) == []


def test_noalloc_header_declares_the_definition():
    """The C declaration in gae_noalloc.h (which callers and the GPU test's ctypes binding read) has the parameter
    types of the definition in gae_noalloc.cu."""
    def params(path):
        text = (CSRC / path).read_text()
        decl = re.search(r"int\s+rlb_gae_advantages_noalloc\s*\(([^)]*)\)", text).group(1)
        return [" ".join(p.split()[:-1]).replace(" *", "*") for p in decl.split(",")]

    assert params("gae_noalloc.h") == params("gae_noalloc.cu")
    assert '#include "gae_noalloc.h"' in (CSRC / "gae_noalloc.cu").read_text()


def test_dependent_launches_wait_before_touching_memory():
    """Every kernel launched with programmatic stream serialization waits for the previous kernel before anything
    else; the GEMM waits before it allocates TMEM and lets dependents start only after it holds its TMEM (so a
    dependent waiting on it never holds TMEM this grid needs)."""
    srcs = {p: p.read_text() for p in CSRC.glob("*.cu")}
    launched = set()
    for text in srcs.values():
        launched.update(re.findall(r"launch_pdl\((\w+)", text))
    assert {"prep_obs_kernel", "gather_minibatch_kernel", "rnn_cell_bwd_kernel"} <= launched
    for name in launched:
        bodies = [t[m.end():] for t in srcs.values()
                  for m in re.finditer(r"__global__ void[^;{]*?\b" + name + r"\s*\([^{]*\{", t)]
        assert bodies, name
        for body in bodies:
            first = body.strip().splitlines()[0]
            assert first.startswith("griddep_wait();"), (name, first)
    gemm = srcs[CSRC / "gemm_tcgen05.cu"]
    kernel = gemm[gemm.index("gemm_tc_kernel(const __grid_constant__"):]
    i_wait, i_alloc, i_trigger = (kernel.index("griddep_wait();"), kernel.index("tmem_alloc(tmem_slot"),
                                  kernel.index("griddep_launch_dependents();"))
    assert i_wait < i_alloc < i_trigger
    assert "cudaLaunchKernelEx" in gemm
