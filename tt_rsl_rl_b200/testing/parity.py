"""Comparison of a kernel's output with its fp32 reference.

:func:`compare` reports the relative Frobenius error, the largest absolute and relative errors (relative over
elements whose reference magnitude exceeds ``rel_floor``), the largest fp32 ULP distance, the Pearson correlation and
the worst element; :data:`TOLERANCES` names the bounds the tests use per kind of computation, so a tolerance is set in
one place and its reason is written next to it. The reference plugin keeps the same kind of registry
(``rsl_rl_tt/testing/parity.py:17-194``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Tol:
    rel_fro: float = 1e-6  # ||a - e||_F / ||e||_F
    max_abs: float | None = None  # max |a - e| (None: not checked)
    pcc_min: float | None = None  # Pearson correlation lower bound
    rel_floor: float = 1e-6  # max_rel only over |e| > rel_floor
    why: str = ""


TOLERANCES: dict[str, Tol] = {
    # bf16 operands (8-bit mantissa), fp32 accumulation over K <= 1024: relative error ~ 2^-8 / sqrt-ish growth
    "gemm_bf16": Tol(rel_fro=1e-2, pcc_min=0.9999, why="bf16 operands, fp32 TMEM accumulation"),
    # gradients of the head written as bf16 (the GEMM operand of the backward pass)
    "grad_bf16": Tol(rel_fro=1e-2, pcc_min=0.9999, why="bf16-rounded output gradients"),
    # fp32 elementwise kernels with the same formula as the reference (rounding-order differences only)
    "fp32_elementwise": Tol(rel_fro=1e-5, why="same fp32 formula, different evaluation order"),
    # fp64-partial reductions (GAE, normaliser moments)
    "fp64_reduced": Tol(rel_fro=1e-6, why="fp64 partial sums"),
    # whole-update function-space deviation, relative to the size of the update (bf16 forward/backward)
    "update_function_space": Tol(rel_fro=0.15, why="one PPO update on bf16 GEMMs vs the fp32 PyTorch path"),
}


@dataclass
class Report:
    rel_fro: float
    max_abs: float
    max_rel: float
    max_ulp: int
    pcc: float
    worst_index: tuple
    worst_actual: float
    worst_expected: float
    ok: bool
    tol: Tol

    def __str__(self) -> str:
        return (f"rel_fro={self.rel_fro:.3e} max_abs={self.max_abs:.3e} max_rel={self.max_rel:.3e} "
                f"max_ulp={self.max_ulp} pcc={self.pcc:.6f} worst{self.worst_index}: actual={self.worst_actual:.6g} "
                f"expected={self.worst_expected:.6g} [{'ok' if self.ok else 'FAIL'} vs {self.tol}]")


def _ulp_distance(a: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
    """Distance in fp32 units in the last place (monotone integer mapping of the float bit patterns)."""
    ai = a.float().contiguous().view(torch.int32).long()
    ei = e.float().contiguous().view(torch.int32).long()
    ai = torch.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    ei = torch.where(ei < 0, -(ei & 0x7FFFFFFF), ei)
    return (ai - ei).abs()


def compare(actual: torch.Tensor, expected: torch.Tensor, tol: Tol | str = "fp32_elementwise") -> Report:
    if isinstance(tol, str):
        tol = TOLERANCES[tol]
    a = actual.detach().double().reshape(-1).cpu()
    e = expected.detach().double().reshape(-1).cpu()
    if a.shape != e.shape:
        raise ValueError(f"shape mismatch: {tuple(actual.shape)} vs {tuple(expected.shape)}")
    diff = (a - e).abs()
    denom = e.norm().item()
    rel_fro = (a - e).norm().item() / denom if denom > 0 else diff.max().item()
    mask = e.abs() > tol.rel_floor
    max_rel = (diff[mask] / e.abs()[mask]).max().item() if bool(mask.any()) else 0.0
    if a.numel() > 1 and float(a.std()) > 0 and float(e.std()) > 0:
        pcc = float(torch.corrcoef(torch.stack([a, e]))[0, 1])
    else:
        pcc = 1.0 if torch.equal(a, e) else 0.0
    w = int(diff.argmax()) if diff.numel() else 0
    idx = tuple(int(i) for i in torch.unravel_index(torch.tensor(w), tuple(actual.shape))) if diff.numel() else ()
    ok = rel_fro <= tol.rel_fro
    if tol.max_abs is not None:
        ok = ok and float(diff.max()) <= tol.max_abs
    if tol.pcc_min is not None:
        ok = ok and pcc >= tol.pcc_min
    return Report(rel_fro=rel_fro, max_abs=float(diff.max()) if diff.numel() else 0.0, max_rel=max_rel,
                  max_ulp=int(_ulp_distance(actual.reshape(-1).cpu(), expected.reshape(-1).cpu()).max())
                  if diff.numel() else 0,
                  pcc=pcc, worst_index=idx, worst_actual=float(a[w]) if diff.numel() else 0.0,
                  worst_expected=float(e[w]) if diff.numel() else 0.0, ok=ok, tol=tol)


def assert_parity(actual: torch.Tensor, expected: torch.Tensor, tol: Tol | str = "fp32_elementwise",
                  what: str = "") -> Report:
    rep = compare(actual, expected, tol)
    if not rep.ok:
        raise AssertionError(f"{what}: {rep}")
    return rep
