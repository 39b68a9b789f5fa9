"""Native-module surface of ``pytorch_opt.ops`` on the sm_100a library.

The reference's ops layer (``pytorch_opt/ops/__init__.py:58-84``) calls a
compiled module with four positional functions, bound in
``pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:103-111``:

    inverse_matrix_root(A, p, damping, method, root_f64, max_iter, tol) -> Tensor
    newton_schulz_orthogonalize(G, steps, a, b, c, eps) -> Tensor
    kron_factor_update_(L, R, G, beta2) -> None       (mutates L and R)
    precond_apply_two_sided(L_root, G, R_root) -> Tensor

This module exports exactly those, with the same argument meaning and the
same error type for bad arguments (``RuntimeError``, as ``TORCH_CHECK``
raises), implemented through the C ABI of ``libpytorch_opt_b200.so``. It is
the object ``pytorch_opt.ops.native_build.load()`` returns once this package
is plugged in as the reference's native backend. It serves CUDA tensors only: there is no
CPU code path here and no silent fallback.

Extra entry points used by the optimizers' hot paths:
``kron_syrk_ema_`` (KFAC factor statistics with the EMA fused),
``damped_inverse`` (KFAC's ``(F + gamma I)^-1`` by the Newton kernel) and
``newton_schulz_batched`` (many matrices in few launches).
"""

from __future__ import annotations

import math

import torch

from . import _lib

_METHODS = ("auto", "eigh", "newton")
_NS_DTYPES = (torch.float32, torch.bfloat16, torch.float16, torch.float64)


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise RuntimeError(f"expected a tensor, got {type(t).__name__}")
        if not t.is_cuda:
            raise RuntimeError("pytorch_opt_b200 runs on CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("all tensors must be on the same CUDA device")
    return dev


def _call(name: str, *args) -> None:
    lib = _lib.load()
    _lib.check(getattr(lib, name)(*args), name)


def _batch_view(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    """Contiguous [batch, rows, cols] view of a (..., rows, cols) tensor."""
    rows, cols = x.shape[-2], x.shape[-1]
    batch = math.prod(x.shape[:-2]) if x.dim() > 2 else 1
    return x.contiguous().reshape(batch, rows, cols), batch, rows, cols


# --------------------------------------------------------------------------
# The four functions of the reference's native module.
# --------------------------------------------------------------------------

def newton_schulz_orthogonalize(G: torch.Tensor, steps: int, a: float, b: float, c: float,
                                eps: float) -> torch.Tensor:
    """Quintic Newton–Schulz polar-factor approximation (reference.py:71-97, cpp:65-81)."""
    if not isinstance(G, torch.Tensor) or G.dim() < 2:
        raise RuntimeError("newton_schulz_orthogonalize expects ndim >= 2")
    dev = _require_cuda(G)
    if G.dtype not in _NS_DTYPES:
        raise RuntimeError(f"newton_schulz_orthogonalize: unsupported dtype {G.dtype}")
    if int(steps) < 0:
        raise RuntimeError("newton_schulz_orthogonalize: steps must be >= 0")
    X, batch, rows, cols = _batch_view(G)
    out = torch.empty_like(X)
    if X.numel() == 0:
        return out.reshape(G.shape)
    with torch.cuda.device(dev):
        lib = _lib.load()
        nbytes = lib.po_ns_workspace_bytes(batch, rows, cols)
        ws = _lib.workspace(nbytes, dev)
        _call("po_newton_schulz", X.data_ptr(), _lib.DTYPE_CODE[X.dtype], batch, rows, cols, cols, rows * cols,
              out.data_ptr(), cols, rows * cols, int(steps), float(a), float(b), float(c), float(eps), -1,
              ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    return out.reshape(G.shape)


def inverse_matrix_root(A: torch.Tensor, p: int, damping: float, method: str, root_f64: bool, max_iter: int,
                        tol: float) -> torch.Tensor:
    """(sym(A) + damping I)^(-1/p) (reference.py:43-68, cpp:41-63).

    ``method="newton"`` runs the tensor-core coupled Newton kernel.
    ``"auto"`` and ``"eigh"`` keep the reference's eigendecomposition route
    (``torch.linalg.eigh`` on the GPU, in fp64 when ``root_f64``).
    """
    if int(p) != p or int(p) < 1:
        raise RuntimeError(f"p must be a positive integer, got {p}")
    if method not in _METHODS:
        raise RuntimeError(f"method must be auto|eigh|newton, got {method}")
    if not isinstance(A, torch.Tensor) or A.dim() < 2 or A.shape[-1] != A.shape[-2]:
        raise RuntimeError("inverse_matrix_root expects square matrices (..., d, d)")
    dev = _require_cuda(A)
    p = int(p)
    if method != "newton":
        return _eigh_root(A, p, float(damping), bool(root_f64))
    orig = A.dtype
    work = A if A.dtype in (torch.float32, torch.bfloat16, torch.float64) else A.float()
    X, batch, d, _ = _batch_view(work)
    out = torch.empty_like(X)
    if X.numel() == 0:
        return out.reshape(A.shape).to(orig)
    with torch.cuda.device(dev):
        lib = _lib.load()
        nbytes = lib.po_root_workspace_bytes(batch, d, p)
        ws = _lib.workspace(nbytes, dev)
        _call("po_inverse_root", X.data_ptr(), _lib.DTYPE_CODE[X.dtype], batch, d, d, d * d, out.data_ptr(), d,
              d * d, p, float(damping), int(max_iter), float(tol), None, ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    return out.reshape(A.shape).to(orig)


def kron_factor_update_(L: torch.Tensor, R: torch.Tensor, G: torch.Tensor, beta2: float) -> None:
    """In place: L <- b L + (1-b) G G^T, R <- b R + (1-b) G^T G (reference.py:100-114, cpp:83-94)."""
    if not isinstance(G, torch.Tensor) or G.dim() != 2:
        raise RuntimeError("G must be 2D")
    dev = _require_cuda(L, R, G)
    m, n = G.shape
    if tuple(L.shape) != (m, m) or tuple(R.shape) != (n, n):
        raise RuntimeError(f"factor shapes {tuple(L.shape)}, {tuple(R.shape)} do not match G {tuple(G.shape)}")
    Lw = L if (L.dtype == torch.float32 and L.is_contiguous()) else L.float().contiguous()
    Rw = R if (R.dtype == torch.float32 and R.is_contiguous()) else R.float().contiguous()
    Gw = G if G.dtype in (torch.float32, torch.bfloat16) else G.float()
    Gw = Gw.contiguous()
    if m and n:
        with torch.cuda.device(dev):
            lib = _lib.load()
            code = _lib.DTYPE_CODE[Gw.dtype]
            nbytes = lib.po_kron_workspace_bytes(m, n, code)
            ws = _lib.workspace(nbytes, dev)
            _call("po_kron_factor_update", Lw.data_ptr(), m, Rw.data_ptr(), n, Gw.data_ptr(), code, m, n, n,
                  float(beta2), ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    if Lw is not L:
        L.copy_(Lw)
    if Rw is not R:
        R.copy_(Rw)


def precond_apply_two_sided(L_root: torch.Tensor, G: torch.Tensor, R_root: torch.Tensor) -> torch.Tensor:
    """L_root @ G @ R_root (reference.py:117-121, cpp:96-99)."""
    return _precond(L_root, G, R_root, False)[0]


def rotate_two_sided(QL: torch.Tensor, G: torch.Tensor, QR: torch.Tensor, trans_l: bool = False,
                     trans_r: bool = False) -> torch.Tensor:
    """op(QL) @ G @ op(QR), op = transpose when requested, without transposed
    copies: SOAP's rotations into the factors' eigenbases, ``QL^T G QR``
    (``trans_l``), and back, ``QL G QR^T`` (``trans_r``)
    (``pytorch_opt/optim/soap.py:118-121``)."""
    return _precond(QL, G, QR, False, trans_l, trans_r)[0]


def _precond(L_root, G, R_root, want_norm: bool, trans_l: bool = False, trans_r: bool = False):
    dev = _require_cuda(L_root, G, R_root)
    if G.dim() != 2 or L_root.dim() != 2 or R_root.dim() != 2:
        raise RuntimeError("precond_apply_two_sided expects 2D operands")
    m, n = G.shape
    if tuple(L_root.shape) != (m, m) or tuple(R_root.shape) != (n, n):
        raise RuntimeError("precond_apply_two_sided: shape mismatch")
    dt = G.dtype if G.dtype in (torch.float32, torch.bfloat16) else torch.float32
    Lc, Gc, Rc = (t.to(dt).contiguous() for t in (L_root, G, R_root))
    out = torch.empty(m, n, dtype=dt, device=dev)
    sq = torch.zeros((), dtype=torch.float64, device=dev) if want_norm else None
    if m and n:
        with torch.cuda.device(dev):
            lib = _lib.load()
            code = _lib.DTYPE_CODE[dt]
            nbytes = lib.po_precond_workspace_bytes(m, n, code)
            ws = _lib.workspace(nbytes, dev)
            _call("po_precond_apply_ex", Lc.data_ptr(), m, 1 if trans_l else 0, Gc.data_ptr(), n, Rc.data_ptr(), n,
                  1 if trans_r else 0, out.data_ptr(), n, code, m, n, sq.data_ptr() if want_norm else None,
                  ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    return (out if out.dtype == G.dtype else out.to(G.dtype)), sq


def precond_apply_grafted(L_root: torch.Tensor, G: torch.Tensor, R_root: torch.Tensor,
                          target: torch.Tensor | float) -> tuple[torch.Tensor, torch.Tensor]:
    """Shampoo's preconditioned direction with grafting (``optim/shampoo.py:126-137``).

    Returns ``(P * ratio, ratio)`` with ``P = L_root @ G @ R_root`` and
    ``ratio = target / (||P||_F + 1e-30)``; ``target`` is the grafted norm
    (``||G||`` for "sgd", the AdaGrad direction's norm for "adagrad"). The
    norm comes from the product's epilogue, and ``ratio`` stays a device
    scalar (the reference reads it back with ``float()``).
    """
    P, sq = _precond(L_root, G, R_root, True)
    ratio = (torch.as_tensor(target, dtype=torch.float64, device=P.device) / (sq.sqrt() + 1e-30))
    return P.mul_(ratio.to(P.dtype)), ratio


# --------------------------------------------------------------------------
# Extra hot-path entry points.
# --------------------------------------------------------------------------

def kron_syrk_ema_(F: torch.Tensor, X: torch.Tensor, alpha: float, beta: float, first: bool,
                   trace: torch.Tensor | None = None) -> torch.Tensor:
    """In place: F <- alpha X^T X when ``first`` else beta F + (1 - beta) alpha X^T X.

    The KFAC factor statistic of ``pytorch_opt/curvature/kron.py:105-113``
    (A = a^T a / n: alpha = 1/n; G = ghat^T ghat / n with ghat = n g:
    alpha = n, applied to g) with the EMA of ``kron.py:95-103``.
    ``trace``: optional fp64 CUDA scalar (a 0-d or 1-element view) that
    receives tr(F) of the updated factor, summed by the product's epilogue.
    """
    dev = _require_cuda(F, X)
    if X.dim() != 2 or F.dim() != 2 or F.shape[0] != F.shape[1] or F.shape[0] != X.shape[1]:
        raise RuntimeError("kron_syrk_ema_: expects X (rows, d) and F (d, d)")
    if F.dtype != torch.float32 or not F.is_contiguous():
        raise RuntimeError("kron_syrk_ema_: F must be a contiguous fp32 tensor")
    Xw = (X if X.dtype in (torch.float32, torch.bfloat16) else X.float()).contiguous()
    rows, d = Xw.shape
    with torch.cuda.device(dev):
        lib = _lib.load()
        code = _lib.DTYPE_CODE[Xw.dtype]
        nbytes = lib.po_syrk_workspace_bytes(rows, d, code)
        ws = _lib.workspace(nbytes, dev)
        tptr = None
        if trace is not None:
            if trace.dtype != torch.float64 or not trace.is_cuda or trace.numel() != 1:
                raise RuntimeError("kron_syrk_ema_: trace must be a one-element fp64 CUDA tensor")
            tptr = trace.data_ptr()
        _call("po_syrk_ema", F.data_ptr(), d, d, Xw.data_ptr(), code, rows, d, float(alpha), float(beta),
              1 if first else 0, tptr, ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    return F


def damped_inverse(F: torch.Tensor, gamma: float, max_iter: int = 100, tol: float = 1e-10) -> torch.Tensor:
    """(sym(F) + gamma I)^-1 by the coupled Newton kernel with p = 1.

    Tensor-core replacement for the fp64 ``eigh`` inverse of
    ``pytorch_opt/optim/kfac.py:134-138``.
    """
    return inverse_matrix_root(F, 1, gamma, "newton", True, max_iter, tol)


def kfac_factored_damping(A: torch.Tensor, G: torch.Tensor, damping: float,
                          traces: torch.Tensor | None = None) -> tuple[float, float]:
    """KFAC's pi-split of the damping (``pytorch_opt/curvature/damping.py:10-25``).

    pi = sqrt((tr(A)/dim A) / (tr(G)/dim G)) (pi = 1 when either mean is not
    finite and positive); returns (pi sqrt(damping), sqrt(damping) / pi).
    ``traces``: optional fp64 CUDA tensor [tr(A), tr(G)], e.g. written by
    ``kron_syrk_ema_(..., trace=traces[0])``; otherwise both diagonals are
    summed on the device. Either way the host reads the two traces once (the
    reference reads each with its own ``float()``).
    """
    if traces is None:
        traces = torch.stack([A.diagonal(dim1=-2, dim2=-1).sum().double(), G.diagonal(dim1=-2, dim2=-1).sum().double()])
    tr_a, tr_g = traces.tolist()
    nu_a = tr_a / A.shape[-1]
    nu_g = tr_g / G.shape[-1]
    if not (math.isfinite(nu_a) and math.isfinite(nu_g)) or nu_a <= 0 or nu_g <= 0:
        pi = 1.0
    else:
        pi = math.sqrt(nu_a / nu_g)
    sq = math.sqrt(damping)
    return pi * sq, sq / pi


class _no_tf32:
    """fp32 torch products without TF32 inside the block."""

    def __enter__(self):
        self.old = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.old


def _top_eigenvalue(F: torch.Tensor, block: int = 16, steps: int = 16, seed: int = 0) -> float:
    """Largest eigenvalue of a symmetric matrix by block Krylov (Rayleigh-Ritz
    on span{Q, FQ, ..., F^(steps-1) Q}, Q a seeded random d x block block):
    a lower bound within ~1e-4 relative of the exact value on the spectra of
    KFAC factors (dense Marchenko-Pastur-like edges)."""
    d = F.shape[-1]
    Ff = F.float()
    g = torch.Generator(device=F.device).manual_seed(seed)
    Q = torch.linalg.qr(torch.randn(d, block, generator=g, device=F.device))[0]
    basis = [Q]
    with _no_tf32():
        for _ in range(steps - 1):
            W = Ff @ basis[-1]
            Qa = torch.cat(basis, 1)
            W = W - Qa @ (Qa.mT @ W)
            W = W - Qa @ (Qa.mT @ W)  # second pass keeps the basis orthogonal in fp32
            basis.append(torch.linalg.qr(W)[0])
        Qa = torch.cat(basis, 1)
        T = (Qa.mT @ (Ff @ Qa)).double()
    return float(torch.linalg.eigvalsh(0.5 * (T + T.mT)).max())


def kfac_damped_inverse(F: torch.Tensor, gamma: float, max_iter: int = 100,
                        tol: float = 1e-10) -> tuple[torch.Tensor, float]:
    """``KFAC._damped_inverse`` (``pytorch_opt/optim/kfac.py:134-138``): returns
    ``((F + gamma I)^-1, cond)`` with cond = (lambda_max + gamma) /
    (lambda_min + gamma), F's dtype kept.

    The inverse is the tensor-core coupled Newton iteration with p = 1
    (``damped_inverse``). The reference takes both from an fp64 ``eigh``;
    here cond = ||F + gamma I||_2 * ||inverse||_2 with both spectral norms
    from block Krylov on the device (exact ``eigvalsh`` for d <= 512), one
    host read.
    """
    inv = damped_inverse(F, gamma, max_iter, tol)
    d = F.shape[-1]
    if d <= 512:
        ev = torch.linalg.eigvalsh(F.double())
        lo, hi = ev.min() + gamma, ev.max() + gamma
        cond = float(hi / lo.clamp_min(1e-300))
    else:
        cond = (_top_eigenvalue(F) + gamma) * _top_eigenvalue(inv)
    return inv.to(F.dtype), cond


def matmul(A: torch.Tensor, B: torch.Tensor, trans_a: bool = False, trans_b: bool = False,
           out: torch.Tensor | None = None, alpha: float = 1.0, beta: float = 0.0) -> torch.Tensor:
    """fp32 ``out = alpha op(A) op(B) + beta out`` on the tensor-core product
    (``po_matmul``; op = transpose, read in place). fp32 operands run as
    split-tf32 (fp32-grade), bf16 operands as bf16 products."""
    dev = _require_cuda(A, B)
    dt = A.dtype if A.dtype in (torch.float32, torch.bfloat16) else torch.float32
    Ac, Bc = A.to(dt).contiguous(), B.to(dt).contiguous()
    M, K = (Ac.shape[1], Ac.shape[0]) if trans_a else tuple(Ac.shape)
    N = Bc.shape[0] if trans_b else Bc.shape[1]
    if (Bc.shape[1] if trans_b else Bc.shape[0]) != K:
        raise RuntimeError("matmul: inner dimensions differ")
    if out is None:
        out = torch.zeros(M, N, dtype=torch.float32, device=dev) if beta else \
            torch.empty(M, N, dtype=torch.float32, device=dev)
    elif out.dtype != torch.float32 or tuple(out.shape) != (M, N) or not out.is_contiguous():
        raise RuntimeError("matmul: out must be a contiguous fp32 M x N tensor")
    if M and N and K:
        with torch.cuda.device(dev):
            lib = _lib.load()
            code = _lib.DTYPE_CODE[dt]
            prec = 2 if dt == torch.float32 else 0
            nbytes = lib.po_matmul_workspace_bytes(1, M, N, K, code, prec)
            ws = _lib.workspace(nbytes, dev)
            _call("po_matmul", Ac.data_ptr(), Ac.shape[1], Ac.numel(), 1 if trans_a else 0, Bc.data_ptr(),
                  Bc.shape[1], Bc.numel(), 1 if trans_b else 0, out.data_ptr(), N, M * N, code, prec, 1, M, N, K,
                  float(alpha), float(beta), ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    return out


def soap_transport_(V: torch.Tensor, QL_old: torch.Tensor, QL_new: torch.Tensor, QR_old: torch.Tensor,
                    QR_new: torch.Tensor) -> torch.Tensor:
    """SOAP's second-moment transport (``pytorch_opt/optim/soap.py:101-108``),
    in place: ``V <- (C_L o C_L)^T V (C_R o C_R)`` with ``C_L = QL_old^T QL_new``,
    ``C_R = QR_old^T QR_new`` (``po_soap_transport``: two basis-change
    products, a squaring pass and the two-sided apply with the transposed
    left operand read in place)."""
    dev = _require_cuda(V, QL_old, QL_new, QR_old, QR_new)
    m, n = V.shape
    dt = V.dtype
    if dt not in (torch.float32, torch.bfloat16):
        raise RuntimeError("soap_transport_: fp32 or bf16 state")
    for Q, d in ((QL_old, m), (QL_new, m), (QR_old, n), (QR_new, n)):
        if tuple(Q.shape) != (d, d) or Q.dtype != dt:
            raise RuntimeError("soap_transport_: bases must be square, matching V's sides and dtype")
    Vc = V if V.is_contiguous() else V.contiguous()
    Qs = [Q.contiguous() for Q in (QL_old, QL_new, QR_old, QR_new)]
    if m and n:
        with torch.cuda.device(dev):
            lib = _lib.load()
            code = _lib.DTYPE_CODE[dt]
            nbytes = lib.po_soap_transport_workspace_bytes(m, n, code)
            ws = _lib.workspace(nbytes, dev)
            _call("po_soap_transport", Qs[0].data_ptr(), Qs[1].data_ptr(), m, Qs[2].data_ptr(), Qs[3].data_ptr(), n,
                  Vc.data_ptr(), n, code, m, n, ws.data_ptr(), nbytes, _lib.stream_ptr(dev))
    if Vc is not V:
        V.copy_(Vc)
    return V


def _cholesky_qr2(Y: torch.Tensor) -> torch.Tensor:
    """Orthonormal basis of Y's columns, column order kept (the Q of Y = QR):
    CholeskyQR twice, ``Y <- Y R^-1`` with ``R^T R = Y^T Y``; the Gram on the
    tensor cores, the triangular factor and solve by the library. A Gram that
    is not numerically positive definite gets a diagonal shift of 1e-6 of its
    mean diagonal and one more pass (shifted CholeskyQR)."""
    passes, k = 2, 0
    while k < passes:
        C = matmul(Y, Y, trans_a=True)
        C = 0.5 * (C + C.mT)
        R, info = torch.linalg.cholesky_ex(C, upper=True)
        if int(info) != 0:
            shift = 1e-6 * float(C.diagonal().mean().clamp_min(1e-30))
            R = torch.linalg.cholesky(C + shift * torch.eye(C.shape[0], device=C.device), upper=True)
            passes += 1
        Y = torch.linalg.solve_triangular(R, Y, upper=True, left=False)
        k += 1
    return Y


def soap_basis(F: torch.Tensor, Q_old: torch.Tensor | None = None, iters: int = 1, shift: float = 1e-3) -> torch.Tensor:
    """Eigenbasis of a SOAP factor (``pytorch_opt/optim/soap.py:98-99``), columns
    in ascending eigenvalue order like ``eigh``.

    Without ``Q_old`` (the first refresh) it is the reference's own fp64
    ``eigh`` on the device. With it, a warm-started subspace iteration: the
    previous basis sorted by its Rayleigh quotients (descending), then
    ``iters`` times ``Q <- qr((F + s I) Q)`` with ``s = shift * max|lambda|``
    (same eigenvectors; it bounds the Gram's condition for CholeskyQR2), the
    products on the tensor cores; finally the columns sorted by ascending
    Rayleigh quotient. This is the power-iteration refresh of Vyas et al.
    (SOAP, 2024), an approximation of the reference's exact ``eigh``: each
    iteration contracts the angle between eigenvectors i and j by about
    (lambda_j + s) / (lambda_i + s), so directions with well-separated
    eigenvalues converge and those inside clusters stay approximate.
    """
    _require_cuda(F)
    if Q_old is None:
        return torch.linalg.eigh(F.double())[1].to(F.dtype)
    if iters < 1:
        raise ValueError("soap_basis: iters must be >= 1")
    Q = Q_old.float()
    Y = matmul(F, Q)
    lam = (Q * Y).sum(0)
    sigma = shift * float(lam.abs().max().clamp_min(1e-30))
    order = torch.argsort(lam, descending=True)
    Q, Y = Q[:, order].contiguous(), Y[:, order].contiguous()
    for it in range(iters):
        if it:
            Y = matmul(F, Q)
        Q = _cholesky_qr2(Y.add_(Q, alpha=sigma))
    lam = (Q * matmul(F, Q)).sum(0)
    return Q[:, torch.argsort(lam)].to(F.dtype)


def soap_refresh_(st: dict, dtype: torch.dtype, method: str = "eigh", iters: int = 1) -> None:
    """SOAP's basis refresh of one parameter's state (``pytorch_opt/optim/soap.py:96-110``):
    new bases of ``st["L"]``, ``st["R"]`` (``method`` "eigh": the reference's
    fp64 eigh; "subspace": ``soap_basis`` warm-started from the previous
    bases), the rotated second moment transported into them on the
    tensor cores (``soap_transport_``), then the bases replaced."""
    if method not in ("eigh", "subspace"):
        raise ValueError(f"unknown SOAP refresh method {method!r}")
    old_l, old_r = st.get("Q_L"), st.get("Q_R")
    warm = method == "subspace" and old_l is not None
    QL = soap_basis(st["L"], old_l if warm else None, iters).to(dtype)
    QR = soap_basis(st["R"], old_r if warm else None, iters).to(dtype)
    if old_l is not None:
        soap_transport_(st["exp_avg_sq"], old_l, QL, old_r, QR)
    st["Q_L"], st["Q_R"] = QL, QR


def newton_schulz_batched(Gs, steps: int = 5, coeffs=(3.4445, -4.7750, 2.0315), eps: float = 1e-7):
    """Orthogonalise many matrices: a 3-D tensor, or a list grouped by (shape, dtype) into batched launches."""
    a, b, c = coeffs
    if isinstance(Gs, torch.Tensor):
        return newton_schulz_orthogonalize(Gs, steps, a, b, c, eps)
    groups: dict = {}
    for i, g in enumerate(Gs):
        groups.setdefault((tuple(g.shape), g.dtype, g.device), []).append(i)
    out = [None] * len(Gs)
    for (_, _, _), idx in groups.items():
        stacked = torch.stack([Gs[i] for i in idx])
        res = newton_schulz_orthogonalize(stacked, steps, a, b, c, eps)
        for j, i in enumerate(idx):
            out[i] = res[j]
    return out


def _eigh_root(A: torch.Tensor, p: int, damping: float, root_f64: bool) -> torch.Tensor:
    orig = A.dtype
    work = torch.float64 if root_f64 else torch.float32
    M = A.to(work)
    M = 0.5 * (M + M.mT)
    if damping:
        M = M + damping * torch.eye(M.shape[-1], dtype=work, device=M.device).expand_as(M)
    evals, evecs = torch.linalg.eigh(M)
    evals = evals.clamp_min(1e-30)
    root = evecs @ torch.diag_embed(evals.pow(-1.0 / p)) @ evecs.mT
    return (0.5 * (root + root.mT)).to(orig)


def ekfac_precondition(QG: torch.Tensor, QA: torch.Tensor, V: torch.Tensor, scale: torch.Tensor | None,
                       decay: float, damping: float) -> tuple[torch.Tensor, torch.Tensor]:
    """EKFAC's rotated-diagonal preconditioning (``optim/ekfac.py:44-58``).

    ``QG`` (m x m) and ``QA`` (n x n) are the factors' eigenbases, ``V`` the
    m x n gradient, ``scale`` the running second moments of the rotated
    gradient (``None`` on the first call: they start as ``Vt**2``; otherwise
    updated in place with ``decay``). Returns ``(QG (Vt / (scale + damping))
    QA^T, scale)`` in ``V``'s dtype; the work runs in fp32 like the reference
    (which casts ``V`` to the eigenbases' dtype).
    """
    dev = _require_cuda(QG, QA, V)
    if V.dim() != 2 or QG.dim() != 2 or QA.dim() != 2:
        raise RuntimeError("ekfac_precondition expects 2D operands")
    m, n = V.shape
    if tuple(QG.shape) != (m, m) or tuple(QA.shape) != (n, n):
        raise RuntimeError("ekfac_precondition: shape mismatch")
    QGc, QAc, Vc = (t.to(torch.float32).contiguous() for t in (QG, QA, V))
    first = scale is None
    if first:
        scale = torch.empty(m, n, dtype=torch.float32, device=dev)
    elif scale.dtype != torch.float32 or tuple(scale.shape) != (m, n) or not scale.is_contiguous():
        raise RuntimeError("ekfac_precondition: scale must be a contiguous fp32 (m, n) tensor")
    out = torch.empty(m, n, dtype=torch.float32, device=dev)
    if m and n:
        with torch.cuda.device(dev):
            lib = _lib.load()
            nbytes = lib.po_ekfac_workspace_bytes(m, n)
            ws = _lib.workspace(nbytes, dev)
            _call("po_ekfac_precondition", QGc.data_ptr(), m, QAc.data_ptr(), n, Vc.data_ptr(), n, scale.data_ptr(), n,
                  out.data_ptr(), n, m, n, 1 if first else 0, float(decay), float(damping), ws.data_ptr(), nbytes,
                  _lib.stream_ptr(dev))
    return (out if V.dtype == torch.float32 else out.to(V.dtype)), scale

