"""Helpers to import the unmodified reference (upstream rsl_rl) installed in ``baseline/_ref``."""

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
COMPAT_DIR = os.path.join(HERE, "compat")


def reference_available() -> bool:
    return os.path.isdir(os.path.join(REF_DIR, "rsl_rl"))


def add_reference_to_path() -> None:
    """Put the reference install and the tensordict stand-in at the front of ``sys.path``."""
    for p in (COMPAT_DIR, REF_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
