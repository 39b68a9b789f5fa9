"""TEST INFRASTRUCTURE ONLY — numpy restatement of the reference algorithms.

Each function follows the cited file:line of kavinravi/pytorch-opt (paths
relative to that project) and is pinned against the reference's own outputs
by ``tests/test_oracle_golden.py``. Arrays are numpy; bf16 tensors are
represented as float32 arrays holding bf16-representable values, with the
rounding made explicit by ``bf16_round``.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "bf16_round", "newton_schulz", "coupled_newton", "inverse_matrix_root", "kron_factor_update",
    "precond_apply", "kfac_batch_factors_linear", "kfac_update", "kfac_factored_damping",
    "kfac_damped_inverse", "muon_scale", "muon_matrix_step", "root_residual", "soap_bases", "soap_transport",
]


def bf16_round(x) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest, ties to even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32).reshape(a.shape)
    return np.where(nan, np.float32(np.nan), out).astype(np.float32)


def _mT(x: np.ndarray) -> np.ndarray:
    return np.swapaxes(x, -1, -2)


def _sym(A: np.ndarray) -> np.ndarray:
    # pytorch_opt/ops/reference.py:13-14
    return 0.5 * (A + _mT(A))


def newton_schulz(G, steps: int = 5, coeffs=(3.4445, -4.7750, 2.0315), eps: float = 1e-7,
                  out_bf16: bool = False) -> np.ndarray:
    """Quintic Newton–Schulz (pytorch_opt/ops/reference.py:71-97).

    Work dtype fp32 (fp64 for fp64 input, :85); transpose when rows > cols
    (:86-89); divide by (||X||_F + eps) (:90); per step A = X X^T,
    B = b A + c A A, X = a X + B X (:91-94); transpose back; cast to the input
    dtype (:95-97; ``out_bf16`` rounds the result to bf16).
    """
    G = np.asarray(G)
    if G.ndim < 2:
        raise ValueError("newton_schulz_orthogonalize expects a matrix (ndim >= 2)")
    a, b, c = coeffs
    work = np.float64 if G.dtype == np.float64 else np.float32
    X = G.astype(work)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = _mT(X)
    nrm = np.sqrt(np.sum(X.astype(np.float64) ** 2, axis=(-2, -1), keepdims=True)).astype(work)
    X = X / (nrm + work(eps))
    for _ in range(steps):
        A = X @ _mT(X)
        B = work(b) * A + work(c) * (A @ A)
        X = work(a) * X + B @ X
    if transposed:
        X = _mT(X)
    if out_bf16:
        return bf16_round(X)
    return X.astype(G.dtype if G.dtype in (np.float32, np.float64) else np.float32)


def coupled_newton(M: np.ndarray, p: int, max_iter: int = 100, tol: float = 1e-10):
    """Coupled Schur–Newton iteration for M^(-1/p) (pytorch_opt/ops/reference.py:17-40).

    Returns (X, iterations). z = (1+p)/(2||M||_F) (:22-24), X0 = z^(1/p) I,
    M0 = z M (:26-27); per step Mi = (1 - alpha) I + alpha Mk, X <- X Mi,
    Mk <- Mi^p Mk, err = max|Mk - I| (:30-33); if err > 1.2 prev: keep the
    previous X and stop (:34-36); stop when err < tol (:38-39).
    """
    M = np.asarray(M, dtype=np.float64)
    n = M.shape[-1]
    I = np.broadcast_to(np.eye(n), M.shape)
    alpha = -1.0 / p
    fro = np.sqrt(np.sum(M * M, axis=(-2, -1)))
    z = (1.0 + p) / (2.0 * np.maximum(fro, np.finfo(np.float64).tiny))
    z = z.reshape(z.shape + (1, 1))
    X = I * z ** (-alpha)
    Mk = M * z
    prev_err = None
    prev_X = X
    its = 0
    for _ in range(max_iter):
        Mi = (1.0 - alpha) * I + alpha * Mk
        X = X @ Mi
        Mk = np.linalg.matrix_power(Mi, p) @ Mk
        its += 1
        err = np.abs(Mk - I).max()
        if prev_err is not None and err > prev_err * 1.2:
            X = prev_X
            break
        prev_X, prev_err = X, err
        if err < tol:
            break
    return X, its


def inverse_matrix_root(A, p: int, damping: float = 0.0, method: str = "auto", root_f64: bool = True,
                        max_iter: int = 100, tol: float = 1e-10) -> np.ndarray:
    """(sym(A) + damping I)^(-1/p) (pytorch_opt/ops/reference.py:43-68).

    Validates p and method (:53-56), symmetrises in the root dtype, adds
    damping (:58-61); "newton" runs ``coupled_newton``, otherwise eigh with
    eigenvalues clamped at 1e-30 (:64-67); symmetrise, cast back (:68).
    """
    if int(p) != p or p < 1:
        raise ValueError(f"p must be a positive integer, got {p}")
    if method not in ("auto", "eigh", "newton"):
        raise ValueError(f"method must be one of ('auto', 'eigh', 'newton'), got {method!r}")
    A = np.asarray(A)
    orig = A.dtype
    work = np.float64 if root_f64 else np.float32
    M = _sym(A.astype(work))
    if damping:
        M = M + work(damping) * np.broadcast_to(np.eye(M.shape[-1], dtype=work), M.shape)
    if method == "newton":
        root = coupled_newton(M, int(p), max_iter, tol)[0]
    else:
        evals, evecs = np.linalg.eigh(M)
        evals = np.maximum(evals, 1e-30)
        root = (evecs * evals[..., None, :] ** (-1.0 / p)) @ _mT(evecs)
    return _sym(root).astype(orig)


def kron_factor_update(L, R, G, beta2: float = 1.0):
    """Kronecker factor update (pytorch_opt/ops/reference.py:100-114); returns new (L, R).

    L <- L + G G^T, R <- R + G^T G when beta2 == 1, else
    L <- beta2 L + (1 - beta2) G G^T (same for R).
    """
    G = np.asarray(G)
    if G.ndim != 2:
        raise ValueError(f"G must be 2D, got shape {tuple(G.shape)}")
    dt = np.asarray(L).dtype
    GGt = (G @ G.T).astype(dt)
    GtG = (G.T @ G).astype(dt)
    if beta2 == 1.0:
        return np.asarray(L) + GGt, np.asarray(R) + GtG
    return (dt.type(beta2) * np.asarray(L) + dt.type(1.0 - beta2) * GGt,
            dt.type(beta2) * np.asarray(R) + dt.type(1.0 - beta2) * GtG)


def precond_apply(L_root, G, R_root) -> np.ndarray:
    """L_root @ G @ R_root (pytorch_opt/ops/reference.py:117-121)."""
    return np.asarray(L_root) @ np.asarray(G) @ np.asarray(R_root)


def kfac_batch_factors_linear(a, g, include_bias: bool = False):
    """KFAC factors of one nn.Linear batch (pytorch_opt/curvature/kron.py:105-113).

    a2, g2 flattened to rows (:107-108), n = rows, ghat = n g2 (:109-110),
    optional bias column of ones (:111-112), A = a2^T a2 / n,
    G = ghat^T ghat / n (:113). Computed in the input precision (fp32).
    """
    a2 = np.asarray(a).reshape(-1, np.asarray(a).shape[-1])
    g2 = np.asarray(g).reshape(-1, np.asarray(g).shape[-1])
    n = a2.shape[0]
    ghat = g2 * a2.dtype.type(n)
    if include_bias:
        a2 = np.concatenate([a2, np.ones((n, 1), dtype=a2.dtype)], axis=1)
    return (a2.T @ a2) / a2.dtype.type(n), (ghat.T @ ghat) / a2.dtype.type(n)


def kfac_update(F, F_b, ema_decay, count: int = 0):
    """Factor accumulation (pytorch_opt/curvature/kron.py:95-103).

    First call (F is None) clones; with ema_decay None a running mean over
    `count` completed updates; else F <- ema F + (1 - ema) F_b.
    """
    if F is None:
        return np.array(F_b, copy=True)
    dt = np.asarray(F).dtype.type
    if ema_decay is None:
        return np.asarray(F) * dt(count / (count + 1)) + np.asarray(F_b) * dt(1.0 / (count + 1))
    return np.asarray(F) * dt(ema_decay) + np.asarray(F_b) * dt(1.0 - ema_decay)


def kfac_factored_damping(A, G, damping: float):
    """pi-split damping (pytorch_opt/curvature/damping.py:10-25): (gamma_A, gamma_G)."""
    tr_a = float(np.trace(np.asarray(A)))
    tr_g = float(np.trace(np.asarray(G)))
    nu_a = tr_a / np.asarray(A).shape[-1]
    nu_g = tr_g / np.asarray(G).shape[-1]
    if not (math.isfinite(nu_a) and math.isfinite(nu_g)) or nu_a <= 0 or nu_g <= 0:
        pi = 1.0
    else:
        pi = math.sqrt(nu_a / nu_g)
    sq = math.sqrt(damping)
    return pi * sq, sq / pi


def kfac_damped_inverse(F, gamma: float):
    """(F + gamma I)^-1 by fp64 eigh, and its condition number (pytorch_opt/optim/kfac.py:134-138)."""
    F = np.asarray(F)
    ev, V = np.linalg.eigh(F.astype(np.float64))
    inv = ((V * (1.0 / (ev + gamma))[None, :]) @ V.T).astype(F.dtype)
    cond = float((ev.max() + gamma) / max(float(ev.min()) + gamma, 1e-300))
    return inv, cond


def ekfac_precondition(QG, QA, V, scale, decay: float, damping: float):
    """EKFAC's rotated-diagonal preconditioning (pytorch_opt/optim/ekfac.py:44-58).

    Vt = QG^T V QA (:51, in the eigenbases' dtype); the running second
    moments start as Vt^2 (:53-55) or take decay*s + (1-decay)*Vt^2 (:57);
    returns (QG (Vt / (s + damping)) QA^T, s) (:58). ``scale`` None = first
    call. Computed in the eigenbases' dtype (fp32 here) like the reference.
    """
    QG = np.asarray(QG)
    work = QG.dtype
    QA = np.asarray(QA, dtype=work)
    V = np.asarray(V, dtype=work)
    Vt = QG.T @ V @ QA
    sq = Vt * Vt
    if scale is None:
        s = sq.copy()
    else:
        s = (np.asarray(scale, dtype=work) * work.type(decay) + work.type(1.0 - decay) * sq).astype(work)
    return (QG @ (Vt / (s + work.type(damping))) @ QA.T).astype(work), s


def soap_bases(L, R, dtype=np.float32):
    """SOAP's refreshed eigenbases (pytorch_opt/optim/soap.py:98-99): fp64
    eigh, eigenvectors in ascending eigenvalue order, cast to the state dtype."""
    ql = np.linalg.eigh(np.asarray(L, dtype=np.float64))[1].astype(dtype)
    qr = np.linalg.eigh(np.asarray(R, dtype=np.float64))[1].astype(dtype)
    return ql, qr


def soap_transport(V, ql_old, ql_new, qr_old, qr_new) -> np.ndarray:
    """SOAP's second-moment transport on a refresh (pytorch_opt/optim/soap.py:101-108):
    C_L = Q_L_old^T Q_L_new, C_R = Q_R_old^T Q_R_new, V' = (C_L^2)^T V (C_R^2), in fp64."""
    f = lambda x: np.asarray(x, dtype=np.float64)  # noqa: E731
    cl = _mT(f(ql_old)) @ f(ql_new)
    cr = _mT(f(qr_old)) @ f(qr_new)
    return _mT(cl * cl) @ f(V) @ (cr * cr)


def muon_scale(shape, lr_adjust: str = "spectral") -> float:
    """Update scale (pytorch_opt/optim/muon.py:51-58)."""
    m, n = shape[-2], shape[-1]
    if lr_adjust == "spectral":
        return max(1.0, m / n) ** 0.5
    if lr_adjust == "match_rms_adam":
        return 0.2 * max(m, n) ** 0.5
    return 1.0


def muon_matrix_step(p, g, buf, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True,
                     ns_steps: int = 5, weight_decay: float = 0.0, lr_adjust: str = "spectral",
                     bf16: bool = True):
    """One Muon update of a matrix parameter (pytorch_opt/optim/muon.py:77-93).

    Returns (p_new, buf_new, O, sum(O^2)). With ``bf16`` every in-place op on
    the bf16 tensors rounds to bf16, as the reference's tensor ops do:
    buf.mul_(mu).add_(g) (:82), u = g.add(buf, alpha=mu) (:83), O = NS(u) cast
    to bf16 (:85), p.mul_(1 - lr wd) (:87-88), p.add_(O, alpha=-lr*scale) (:91).
    torch's CPU ``add(..., alpha=a)`` on a bf16 tensor first rounds ``a`` to
    bf16 (``mul_`` by a scalar does not); the golden vectors show it, and it is
    reproduced here.
    """
    rnd = bf16_round if bf16 else (lambda x: np.asarray(x, dtype=np.float32))
    p = np.asarray(p, dtype=np.float32)
    g = np.asarray(g, dtype=np.float32)
    buf = np.asarray(buf, dtype=np.float32)
    buf = rnd(rnd(buf * np.float32(momentum)) + g)
    u = rnd(g + rnd(np.float32(momentum)) * buf) if nesterov else buf
    u2 = u if u.ndim == 2 else u.reshape(u.shape[0], -1)
    O = newton_schulz(u2.astype(np.float32), ns_steps, out_bf16=bf16)
    scale = muon_scale(O.shape, lr_adjust)
    if weight_decay:
        p = rnd(p * np.float32(1.0 - lr * weight_decay))
    eff = lr * scale
    p = rnd(p + rnd(np.float32(-eff)) * O.reshape(p.shape))
    return p, buf, O, float(np.sum(O.astype(np.float64) ** 2))


def root_residual(X, A, p: int, damping: float = 0.0) -> float:
    """||X^p (A + damping I) - I||_F / sqrt(d), computed in fp64 (the parity metric for roots)."""
    X = np.asarray(X, dtype=np.float64)
    A = np.asarray(A, dtype=np.float64)
    d = A.shape[-1]
    M = A + damping * np.eye(d)
    R = np.linalg.matrix_power(X, p) @ M - np.eye(d)
    return float(np.sqrt(np.sum(R * R, axis=(-2, -1))).max() / math.sqrt(d))
