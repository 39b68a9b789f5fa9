"""TEST INFRASTRUCTURE ONLY — torch restatement of the reference algorithms,
used as the checker at full problem size.

The numpy oracle (``oracle.ops_np``) is the checker for sizes the host
finishes in seconds. The configurations the benchmark runs on (Llama-3-8B
Newton–Schulz shapes up to 14336 x 4096, 4096^2 roots and KFAC factors from
8192 rows) take minutes there, so the parity tests evaluate the same
algorithm with torch on the GPU: fp32 without TF32 for Newton–Schulz (what
the reference computes, ``reference.py:85``), fp64 for the roots and factor
statistics. These functions are pinned against the reference's own outputs:
golden vectors at small sizes and two-sided sketches of the reference's
full-size outputs (``tests/golden/full_size.npz``, written by
``tests/golden/make_full_size.py``), checked by ``tests/test_oracle_golden.py``
and ``tests/test_gpu_full_size.py``.
"""

from __future__ import annotations

import contextlib

import torch


@contextlib.contextmanager
def exact_fp32_matmul():
    """Disable TF32 for torch products (the reference's fp32 semantics)."""
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def newton_schulz(G: torch.Tensor, steps: int = 5, coeffs=(3.4445, -4.7750, 2.0315),
                  eps: float = 1e-7) -> torch.Tensor:
    """Quintic Newton–Schulz, ``pytorch_opt/ops/reference.py:71-97``.

    Work dtype fp32 (fp64 for fp64 input, :85); transpose when rows > cols
    (:86-89); divide by (||X||_F + eps) (:90); per step A = X X^T,
    B = b A + c A A, X = a X + B X (:91-94); transpose back and cast to the
    input dtype (:95-97). Run under ``exact_fp32_matmul()``.
    """
    a, b, c = coeffs
    work = torch.float64 if G.dtype == torch.float64 else torch.float32
    X = G.to(work)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = X.mT
    X = X / (torch.linalg.matrix_norm(X, ord="fro", keepdim=True) + eps)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if transposed:
        X = X.mT
    return X.to(G.dtype)


def coupled_newton(M: torch.Tensor, p: int, max_iter: int = 100, tol: float = 1e-10):
    """Coupled Newton iteration for M^(-1/p), ``pytorch_opt/ops/reference.py:17-40``.

    Returns ``(X, iterations)`` for one matrix (fp64). z = (1+p)/(2||M||_F)
    (:22-24), X0 = z^(1/p) I, M0 = z M (:25-26); per step Mi = (1-alpha) I +
    alpha Mk, X <- X Mi, Mk <- Mi^p Mk, err = max|Mk - I| (:29-33); if
    err > 1.2 prev keep the previous X and stop (:34-36); stop when err < tol
    (:38-39).
    """
    n = M.shape[-1]
    I = torch.eye(n, dtype=M.dtype, device=M.device)
    alpha = -1.0 / p
    fro = torch.linalg.matrix_norm(M, ord="fro")
    z = (1.0 + p) / (2.0 * fro.clamp_min(torch.finfo(M.dtype).tiny))
    X = I * z.pow(-alpha)
    Mk = M * z
    prev_err = None
    prev_X = X
    its = 0
    for _ in range(max_iter):
        Mi = (1.0 - alpha) * I + alpha * Mk
        X = X @ Mi
        Mk = torch.linalg.matrix_power(Mi, p) @ Mk
        its += 1
        err = float((Mk - I).abs().amax())
        if prev_err is not None and err > prev_err * 1.2:
            X = prev_X
            break
        prev_X, prev_err = X, err
        if err < tol:
            break
    return X, its


def inverse_root_newton(A: torch.Tensor, p: int, damping: float = 0.0, max_iter: int = 100, tol: float = 1e-10):
    """``inverse_matrix_root(A, p, damping, method="newton")`` in fp64,
    ``pytorch_opt/ops/reference.py:58-63,68``: symmetrise, damp, iterate,
    symmetrise. Returns ``(X, iterations)``."""
    M = A.to(torch.float64)
    M = 0.5 * (M + M.mT)
    if damping:
        M = M + damping * torch.eye(M.shape[-1], dtype=M.dtype, device=M.device)
    X, its = coupled_newton(M, p, max_iter, tol)
    return 0.5 * (X + X.mT), its


def root_residual(X: torch.Tensor, A: torch.Tensor, p: int, damping: float) -> float:
    """||X^p (A + damping I) - I||_F / sqrt(d), evaluated in fp64."""
    Xd = X.to(torch.float64)
    d = Xd.shape[-1]
    I = torch.eye(d, dtype=torch.float64, device=Xd.device)
    R = torch.linalg.matrix_power(Xd, p) @ (A.to(torch.float64) + damping * I) - I
    return float(R.norm() / d ** 0.5)


def kron_batch_factor(X: torch.Tensor, alpha: float) -> torch.Tensor:
    """alpha * X^T X in fp64 (``pytorch_opt/curvature/kron.py:105-113``:
    A = a^T a / n with alpha = 1/n; G = ghat^T ghat / n, ghat = n g, i.e.
    alpha = n applied to g)."""
    Xd = X.to(torch.float64)
    return alpha * (Xd.mT @ Xd)


def kfac_update(F, F_batch: torch.Tensor, beta: float) -> torch.Tensor:
    """``KronTracker._update`` (``pytorch_opt/curvature/kron.py:95-103``):
    the first call clones, later calls F <- beta F + (1 - beta) F_batch."""
    if F is None:
        return F_batch.clone()
    return beta * F + (1.0 - beta) * F_batch


def damped_inverse(F: torch.Tensor, gamma: float):
    """``KFAC._damped_inverse`` (``pytorch_opt/optim/kfac.py:134-138``):
    fp64 eigh of F (its lower triangle), V diag(1/(ev + gamma)) V^T and
    cond = (max(ev) + gamma) / max(min(ev) + gamma, 1e-300). Returns
    (inverse in fp64, cond)."""
    ev, V = torch.linalg.eigh(F.to(torch.float64))
    inv = (V * (1.0 / (ev + gamma))) @ V.mT
    cond = float((ev.max() + gamma) / max(float(ev.min()) + gamma, 1e-300))
    return inv, cond


def two_sided_sketch(X: torch.Tensor, left_seed: int, right_seed: int, k: int = 32) -> torch.Tensor:
    """L^T X R (fp64, k x k) with L (rows x k) and R (cols x k) i.i.d. N(0,1)
    drawn on the CPU from the given seeds: a size-independent fingerprint of
    X. For two matrices, ||sketch(X) - sketch(Y)|| / ||sketch(Y)|| estimates
    ||X - Y||_F / ||Y||_F (to ~10 % at k = 32)."""
    rows, cols = X.shape[-2], X.shape[-1]
    L = torch.randn(rows, k, generator=torch.Generator().manual_seed(left_seed), dtype=torch.float64)
    R = torch.randn(cols, k, generator=torch.Generator().manual_seed(right_seed), dtype=torch.float64)
    L, R = L.to(X.device), R.to(X.device)
    return L.mT @ X.to(torch.float64) @ R
