"""TEST INFRASTRUCTURE ONLY — load the reference's compiled ATen ops from ``oracle/_ref/``.

Returns the pybind module built by ``oracle/build_ref.py`` from the
reference's ``pytorch_opt_ops.cpp`` (functions ``inverse_matrix_root``,
``newton_schulz_orthogonalize``, ``kron_factor_update_``,
``precond_apply_two_sided``), or None when it has not been built.
"""

from __future__ import annotations

import importlib.util
import os

from .build_ref import MODULE, target_path

_MOD = None


def load():
    global _MOD
    if _MOD is not None:
        return _MOD
    path = target_path()
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(MODULE, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    _MOD = mod
    return mod
