"""Test tooling: numerical parity (tolerance registry and comparison metrics, ``parity``), reference training runs on
the seeded test environments for this framework or upstream rsl_rl (``reference``), golden learning curves and their
acceptance rule (``golden``), and mirror functions of the test environments (``symmetry``)."""

from .parity import TOLERANCES, Report, Tol, assert_parity, compare

__all__ = ["TOLERANCES", "Report", "Tol", "assert_parity", "compare"]
