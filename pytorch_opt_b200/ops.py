"""``pytorch_opt.ops`` public surface on the B200-native library.

Same names, signatures, defaults and argument checks as the reference's
``pytorch_opt/ops/__init__.py:21-88`` and ``pytorch_opt/ops/reference.py``:

    inverse_matrix_root(A, p, damping=0.0, method="auto", root_dtype=torch.float64,
                        max_iter=100, tol=1e-10)
    newton_schulz_orthogonalize(G, steps=5, coeffs=(3.4445, -4.7750, 2.0315), eps=1e-7)
    kron_factor_update_(L, R, G, beta2=1.0) -> (L, R)
    precond_apply_two_sided(L_root, G, R_root)
    load_native(verbose=False) -> bool      (never raises; warns RuntimeWarning)
    native_available() -> bool
    set_backend(name) / get_backend()      ("auto" | "native" | "reference")

Argument errors raise ``ValueError`` as in ``reference.py:53-56, 82-83,
104-105``. This package is the native backend only: the pure-torch
"reference" backend stays in ``pytorch_opt.ops.reference``, so selecting it
here raises, and an op called while the library cannot be loaded raises
instead of falling back to another implementation.
"""

from __future__ import annotations

import os
import warnings

import torch

from . import _lib, native

_VALID_BACKENDS = ("auto", "native", "reference")
_VALID_ROOT_METHODS = ("auto", "eigh", "newton")
_BACKEND = "auto"
_LOADED = False


def get_backend() -> str:
    return _BACKEND


def native_available() -> bool:
    return _LOADED


def set_backend(name: str) -> None:
    global _BACKEND
    if name not in _VALID_BACKENDS:
        raise ValueError(f"backend must be one of {_VALID_BACKENDS}, got {name!r}")
    if name == "native" and not _LOADED:
        raise RuntimeError("native backend not loaded; call pytorch_opt_b200.ops.load_native() first")
    if name == "reference":
        raise RuntimeError("pytorch_opt_b200 is the native backend only; the reference backend is "
                           "pytorch_opt.ops.reference")
    _BACKEND = name


def load_native(verbose: bool = False) -> bool:
    """Load ``libpytorch_opt_b200.so``. Returns True on success; never raises."""
    global _LOADED
    if _LOADED:
        return True
    try:
        lib = _lib.load()
        if verbose:
            print(f"pytorch_opt_b200: loaded {_lib.LIB_PATH} ({lib.po_version().decode()})")
        _LOADED = True
        return True
    except Exception as e:  # report, never break import
        warnings.warn(f"pytorch_opt_b200: native library unavailable ({type(e).__name__}: {e})",
                      RuntimeWarning, stacklevel=2)
        return False


def _native():
    if not _LOADED and not load_native():
        raise RuntimeError("pytorch_opt_b200: the native library could not be loaded (no fallback exists)")
    return native


def inverse_matrix_root(A, p, damping=0.0, method="auto", root_dtype=torch.float64, max_iter=100, tol=1e-10):
    """(A + damping*I)^(-1/p) for symmetric PSD A, batched over leading dims."""
    if int(p) != p or p < 1:
        raise ValueError(f"p must be a positive integer, got {p}")
    if method not in _VALID_ROOT_METHODS:
        raise ValueError(f"method must be one of {_VALID_ROOT_METHODS}, got {method!r}")
    return _native().inverse_matrix_root(A, int(p), float(damping), str(method), root_dtype == torch.float64,
                                         int(max_iter), float(tol))


def newton_schulz_orthogonalize(G, steps=5, coeffs=(3.4445, -4.7750, 2.0315), eps=1e-7):
    """Quintic Newton-Schulz approximation of the orthogonal polar factor of G (batched)."""
    if G.ndim < 2:
        raise ValueError("newton_schulz_orthogonalize expects a matrix (ndim >= 2)")
    a, b, c = coeffs
    return _native().newton_schulz_orthogonalize(G, int(steps), float(a), float(b), float(c), float(eps))


def kron_factor_update_(L, R, G, beta2=1.0):
    """In-place Kronecker factor accumulation: L += G G^T, R += G^T G (or EMA)."""
    if G.ndim != 2:
        raise ValueError(f"G must be 2D, got shape {tuple(G.shape)}")
    _native().kron_factor_update_(L, R, G, float(beta2))
    return L, R


def precond_apply_two_sided(L_root, G, R_root):
    """L_root @ G @ R_root."""
    return _native().precond_apply_two_sided(L_root, G, R_root)


if os.environ.get("PYTORCH_OPT_NATIVE") == "1":
    load_native()
