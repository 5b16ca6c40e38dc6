"""Numerical parity tooling for kernel and engine tests (tolerance registry and comparison metrics)."""

from .parity import TOLERANCES, Report, Tol, assert_parity, compare

__all__ = ["TOLERANCES", "Report", "Tol", "assert_parity", "compare"]
