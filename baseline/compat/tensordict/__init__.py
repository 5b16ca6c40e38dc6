"""Stand-in for the ``tensordict`` package, which this image lacks and which upstream rsl_rl imports.

It exposes the TensorDict class defined in ``tt_rsl_rl_b200/utils/tensordict.py``, loaded directly from that file
(which depends only on torch), so that the unmodified reference can run without importing any of the framework's
models, kernels or engine. Only the benchmark's reference arm and the CPU oracle tests put this directory on
``sys.path``.
"""

import importlib.util
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "..", "..", "..", "tt_rsl_rl_b200", "utils", "tensordict.py")
_spec = importlib.util.spec_from_file_location("_tensordict_standin", os.path.normpath(_SRC))
_mod = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_mod)

TensorDict = _mod.TensorDict

__all__ = ["TensorDict"]
