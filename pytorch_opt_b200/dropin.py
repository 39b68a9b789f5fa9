"""Plug this library into an installed kavinravi/pytorch-opt as its native backend.

``install()`` makes, in the running process, the changes a maintainer would
make in the reference's sources to use the B200 kernels:

* ops layer (``pytorch_opt/ops/__init__.py:21-88``): ``_NATIVE`` becomes
  ``pytorch_opt_b200.native`` (the four positional functions of
  ``pytorch_opt_ops.cpp:103-111``), and the four op wrappers route CUDA
  tensors to it when the backend switch selects the native backend
  (``"auto"`` or ``"native"``) and everything else — CPU tensors, or the
  ``"reference"`` backend — to the reference's own ``ops.reference``
  (the CUDA-only ``_use_native``). Muon (``optim/muon.py:85``), Shampoo
  (``optim/shampoo.py:101,112,115,126``) and SOAP (``optim/soap.py:95``)
  call these wrappers through the module at call time, so they need no change.
* KFAC, whose factor statistics and inverses do not go through ``ops``:
  ``KronTracker._on_grad_out`` (``curvature/kron.py:82-103``) updates the
  factors of CUDA Linear and Conv2d layers with the fused SYRK+EMA kernel
  (first call clones, then EMA or running mean; each factor's trace comes
  from the kernel's epilogue); ``kfac_factored_damping`` as ``optim/kfac.py``
  binds it (:23, used at :153) reads those traces once; ``KFAC._damped_inverse``
  (``optim/kfac.py:134-138``) returns the tensor-core inverse and its
  condition number; ``KFAC._precondition`` (:140-147) runs ``iG @ V @ iA`` on
  the two-sided apply kernel and ``EKFAC._precondition`` (``optim/ekfac.py:44-58``)
  on the rotated-diagonal kernel.
* SOAP: ``SOAP._soap_update`` (``optim/soap.py:47-64``) receives its
  rotations into and out of the factors' eigenbases as the two-sided apply
  kernel with transposed operands read in place (``soap.py:118-121``).
  ``SOAP.step`` (``:66-131``) is restated with its basis refresh
  (``:96-110``) as ``native.soap_refresh_``: the second-moment transport on
  the tensor cores, the bases by the reference's fp64 ``eigh``
  (``soap_refresh="eigh"``, the default) or by the warm-started subspace
  iteration (``"subspace"``, an approximation; ``soap_refresh=None`` keeps
  the reference's step).

Every replacement falls through to the reference's original code for inputs
this library does not serve (CPU tensors, fp64 factors), exactly as the
reference's own dispatch does for its native module. ``uninstall()``
restores the originals.
"""

from __future__ import annotations

import weakref

import torch
from torch import nn
import torch.nn.functional as Fn

from . import native

_SAVED: dict = {}
# id(factor) -> (weakref to the factor, trace buffer, index, factor._version at the update)
_TRACES: dict = {}


def _on_gpu(*ts) -> bool:
    return all(isinstance(t, torch.Tensor) and t.is_cuda for t in ts)


def _record_trace(F: torch.Tensor, buf: torch.Tensor, idx: int) -> None:
    _TRACES[id(F)] = (weakref.ref(F), buf, idx, F._version)


def _trace_of(F: torch.Tensor):
    ent = _TRACES.get(id(F))
    if ent is None:
        return None
    ref, buf, idx, ver = ent
    if ref() is not F or F._version != ver:  # another tensor, or modified since the kernel's update
        return None
    return buf, idx


def _install_ops(ops) -> None:
    ref = ops.reference

    def inverse_matrix_root(A, p, damping=0.0, method="auto", root_dtype=torch.float64, max_iter=100, tol=1e-10):
        if ops._use_native() and _on_gpu(A):
            return ops._NATIVE.inverse_matrix_root(A, int(p), float(damping), str(method),
                                                   root_dtype == torch.float64, int(max_iter), float(tol))
        return ref.inverse_matrix_root(A, p, damping=damping, method=method, root_dtype=root_dtype,
                                       max_iter=max_iter, tol=tol)

    def newton_schulz_orthogonalize(G, steps=5, coeffs=(3.4445, -4.7750, 2.0315), eps=1e-7):
        if ops._use_native() and _on_gpu(G):
            a, b, c = coeffs
            return ops._NATIVE.newton_schulz_orthogonalize(G, int(steps), float(a), float(b), float(c), float(eps))
        return ref.newton_schulz_orthogonalize(G, steps=steps, coeffs=coeffs, eps=eps)

    def kron_factor_update_(L, R, G, beta2=1.0):
        if ops._use_native() and _on_gpu(L, R, G):
            ops._NATIVE.kron_factor_update_(L, R, G, float(beta2))
            return L, R
        return ref.kron_factor_update_(L, R, G, beta2=beta2)

    def precond_apply_two_sided(L_root, G, R_root):
        if ops._use_native() and _on_gpu(L_root, G, R_root):
            return ops._NATIVE.precond_apply_two_sided(L_root, G, R_root)
        return ref.precond_apply_two_sided(L_root, G, R_root)

    _SAVED["ops"] = (ops, {k: getattr(ops, k) for k in ("_NATIVE", "inverse_matrix_root",
                                                         "newton_schulz_orthogonalize", "kron_factor_update_",
                                                         "precond_apply_two_sided")})
    ops._NATIVE = native
    ops.inverse_matrix_root = inverse_matrix_root
    ops.newton_schulz_orthogonalize = newton_schulz_orthogonalize
    ops.kron_factor_update_ = kron_factor_update_
    ops.precond_apply_two_sided = precond_apply_two_sided


def _factor_rows(tracker, module, a: torch.Tensor, g: torch.Tensor):
    """The rows whose Gram matrices are the batch factors of
    ``KronTracker._batch_factors`` (``curvature/kron.py:105-124``):
    returns (rows of a (bias column appended when tracked), alpha_A, rows of
    the output gradients, alpha_G) with A_b = alpha_A a^T a and
    G_b = alpha_G g^T g (ghat = n g / grad_scale folded into alpha_G)."""
    s2 = tracker.grad_scale ** 2
    if isinstance(module, nn.Linear):
        a2 = a.reshape(-1, a.shape[-1])
        g2 = g.reshape(-1, g.shape[-1])
        n = a2.shape[0]
        if tracker.includes_bias(module):
            a2 = torch.cat([a2, a2.new_ones(n, 1)], dim=1)
        return a2, 1.0 / n, g2, n / s2
    B = a.shape[0]
    patches = Fn.unfold(a, module.kernel_size, dilation=module.dilation, padding=module.padding,
                        stride=module.stride)
    L = patches.shape[-1]
    at = patches.permute(0, 2, 1).reshape(B * L, -1)
    if tracker.includes_bias(module):
        at = torch.cat([at, at.new_ones(B * L, 1)], dim=1)
    gt = g.reshape(B, g.shape[1], -1).permute(0, 2, 1).reshape(B * L, -1)
    return at, 1.0 / (B * L), gt, B / (L * s2)


def _install_kfac(pytorch_opt) -> None:
    import importlib
    kron = importlib.import_module(pytorch_opt.__name__ + ".curvature.kron")
    kfac_mod = importlib.import_module(pytorch_opt.__name__ + ".optim.kfac")
    ekfac_mod = importlib.import_module(pytorch_opt.__name__ + ".optim.ekfac")
    KronTracker, KFAC, EKFAC = kron.KronTracker, kfac_mod.KFAC, ekfac_mod.EKFAC
    orig_on_grad = KronTracker._on_grad_out
    orig_damping = kfac_mod.kfac_factored_damping
    orig_inverse = KFAC.__dict__["_damped_inverse"]
    orig_precond = KFAC.__dict__["_precondition"]
    orig_eprecond = EKFAC.__dict__["_precondition"]

    def _on_grad_out(self, module, a, grad_output):
        if not (self.enabled and module.training):
            return
        served = (a.is_cuda and isinstance(module, (nn.Linear, nn.Conv2d))
                  and module.weight.dtype != torch.float64)
        name = self._module_names[module]
        d = self.factors.get(name, {})
        for key in ("A", "G"):
            if key in d and not (d[key].dtype == torch.float32 and d[key].is_contiguous() and d[key].is_cuda):
                served = False  # e.g. restored from a checkpoint in another dtype: the reference's own path
        if not served:
            return orig_on_grad(self, module, a, grad_output)
        with torch.autocast(device_type="cuda", enabled=False):
            ra, alpha_a, rg, alpha_g = _factor_rows(self, module, a, grad_output.detach())
        d = self.factors.setdefault(name, {})
        cnt = self._counts.get(name, 0)
        beta = self.ema_decay if self.ema_decay is not None else cnt / (cnt + 1)
        traces = torch.zeros(2, dtype=torch.float64, device=a.device)
        for i, (key, X, alpha) in enumerate((("A", ra, alpha_a), ("G", rg, alpha_g))):
            first = key not in d
            F = d[key] if not first else torch.empty(X.shape[1], X.shape[1], dtype=torch.float32, device=a.device)
            native.kron_syrk_ema_(F, X, alpha, beta, first, trace=traces[i:i + 1])
            d[key] = F
            _record_trace(F, traces, i)
        self._counts[name] = cnt + 1

    def kfac_factored_damping(A, G, damping):
        if not _on_gpu(A, G):
            return orig_damping(A, G, damping)
        ta, tg = _trace_of(A), _trace_of(G)
        traces = None
        if ta is not None and tg is not None:
            traces = ta[0] if (ta[0] is tg[0] and ta[1] == 0 and tg[1] == 1) else torch.stack(
                [ta[0][ta[1]], tg[0][tg[1]]])
        return native.kfac_factored_damping(A, G, damping, traces)

    def _damped_inverse(F, gamma):
        if not _on_gpu(F):
            return orig_inverse.__func__(F, gamma)
        return native.kfac_damped_inverse(F, gamma)

    def _precondition(self, name, V):
        inv = self._inv.get(name)
        if inv is None or not _on_gpu(inv["iG"], inv["iA"], V) or inv["iG"].dtype != torch.float32:
            return orig_precond(self, name, V)
        with torch.autocast(device_type="cuda", enabled=False):
            return native.precond_apply_two_sided(inv["iG"], V.to(inv["iG"].dtype), inv["iA"]).to(V.dtype)

    def _eprecondition(self, name, V):
        inv = self._inv.get(name)
        if inv is None or not _on_gpu(inv["QG"], inv["QA"], V) or inv["QG"].dtype != torch.float32:
            return orig_eprecond(self, name, V)
        out, self._scales[name] = native.ekfac_precondition(inv["QG"], inv["QA"], V, self._scales.get(name),
                                                            self._scale_decay, self.param_groups[0]["damping"])
        return out.to(V.dtype)

    soap_mod = importlib.import_module(pytorch_opt.__name__ + ".optim.soap")
    SOAP = soap_mod.SOAP
    orig_soap_update = SOAP.__dict__["_soap_update"]

    def _soap_update(p, g, st, group, *, transform, back):
        QL, QR = st.get("Q_L"), st.get("Q_R")
        if QL is not None and _on_gpu(QL, QR, g) and QL.dtype == torch.float32 and g.dtype == torch.float32:
            transform = lambda x: native.rotate_two_sided(QL, x, QR, trans_l=True)  # noqa: E731  QL^T x QR
            back = lambda x: native.rotate_two_sided(QL, x, QR, trans_r=True)  # noqa: E731  QL x QR^T
        return orig_soap_update.__func__(p, g, st, group, transform=transform, back=back)

    _SAVED["kfac"] = [(KronTracker, "_on_grad_out", orig_on_grad), (kfac_mod, "kfac_factored_damping", orig_damping),
                      (KFAC, "_damped_inverse", orig_inverse), (KFAC, "_precondition", orig_precond),
                      (EKFAC, "_precondition", orig_eprecond), (SOAP, "_soap_update", orig_soap_update)]
    SOAP._soap_update = staticmethod(_soap_update)
    KronTracker._on_grad_out = _on_grad_out
    kfac_mod.kfac_factored_damping = kfac_factored_damping
    KFAC._damped_inverse = staticmethod(_damped_inverse)
    KFAC._precondition = _precondition
    EKFAC._precondition = _eprecondition


def _install_soap_step(pytorch_opt, method: str, iters: int) -> None:
    """Restate ``SOAP.step`` (``optim/soap.py:66-131``) with the refresh on this library."""
    import importlib
    soap_mod = importlib.import_module(pytorch_opt.__name__ + ".optim.soap")
    ops = importlib.import_module(pytorch_opt.__name__ + ".ops")
    SOAP = soap_mod.SOAP
    orig_step = SOAP.__dict__["step"]
    timer, matrix_path, adamw_update = soap_mod.StepTimer, soap_mod.matrix_path, soap_mod.adamw_update

    def refresh(p, st):
        """soap.py:96-110: new bases of L and R, the rotated second moment carried into them."""
        if _on_gpu(st["L"], st["R"]) and p.dtype in (torch.float32, torch.bfloat16):
            native.soap_refresh_(st, p.dtype, method, iters)
            return
        QL = torch.linalg.eigh(st["L"].double())[1].to(p.dtype)
        QR = torch.linalg.eigh(st["R"].double())[1].to(p.dtype)
        if "Q_L" in st:
            CL, CR = st["Q_L"].T @ QL, st["Q_R"].T @ QR
            st["exp_avg_sq"] = CL.pow(2).T @ st["exp_avg_sq"] @ CR.pow(2)
        st["Q_L"], st["Q_R"] = QL, QR

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        curvature_ms, stales, n_adamw = 0.0, [], 0
        with timer() as t_all:
            for group in self.param_groups:
                for p in group["params"]:
                    if p.grad is None:
                        continue
                    st = self.state[p]
                    if not matrix_path(p, group):
                        n_adamw += 1
                        adamw_update(p, p.grad, st, group)
                        continue
                    g2 = p.grad.reshape(p.grad.shape[0], -1)
                    m, n = g2.shape
                    if "L" not in st:
                        st.update(L=torch.zeros(m, m, device=p.device, dtype=p.dtype),
                                  R=torch.zeros(n, n, device=p.device, dtype=p.dtype),
                                  exp_avg=torch.zeros_like(g2), exp_avg_sq=torch.zeros_like(g2), step=0, stale=0)
                    ops.kron_factor_update_(st["L"], st["R"], g2, beta2=group["shampoo_beta"])
                    if st["step"] % group["precondition_frequency"] == 0:
                        with timer() as t_c:
                            refresh(p, st)
                        curvature_ms += t_c.ms
                        st["stale"] = 0
                    else:
                        st["stale"] += 1
                    stales.append(st["stale"])
                    QL, QR = st["Q_L"], st["Q_R"]
                    self._soap_update(p.view(m, n), g2, st, group,
                                      transform=lambda x, QL=QL, QR=QR: QL.T @ x @ QR,
                                      back=lambda x, QL=QL, QR=QR: QL @ x @ QR.T)
        self._diag = {"stale_steps": max(stales) if stales else 0, "n_adamw_params": n_adamw,
                      "step_ms": t_all.ms, "curvature_ms": curvature_ms}
        return loss

    _SAVED["soap"] = [(SOAP, "step", orig_step)]
    SOAP.step = step


def install(pytorch_opt=None, kfac: bool = True, soap_refresh: str | None = "eigh", soap_iters: int = 1) -> None:
    """Install this library as ``pytorch_opt``'s native backend (and, with
    ``kfac``, the KFAC and SOAP rewiring). ``pytorch_opt``: the imported
    reference package (imported here when omitted). ``soap_refresh``: the
    SOAP basis refresh (``"eigh"``: the reference's bases, transport on the
    tensor cores; ``"subspace"``: ``native.soap_basis`` warm-started with
    ``soap_iters`` iterations; None: the reference's ``SOAP.step``).
    Idempotent; ``uninstall()`` first to change the options."""
    if pytorch_opt is None:
        import pytorch_opt
    from importlib import import_module
    if soap_refresh not in (None, "eigh", "subspace"):
        raise ValueError(f"unknown soap_refresh {soap_refresh!r}")
    ops = import_module(pytorch_opt.__name__ + ".ops")
    if "ops" not in _SAVED:
        _install_ops(ops)
    if kfac and "kfac" not in _SAVED:
        _install_kfac(pytorch_opt)
        if soap_refresh is not None and "soap" not in _SAVED:
            _install_soap_step(pytorch_opt, soap_refresh, soap_iters)


def uninstall() -> None:
    """Restore the reference's original functions."""
    if "ops" in _SAVED:
        ops, saved = _SAVED.pop("ops")
        for k, v in saved.items():
            setattr(ops, k, v)
    for owner, attr, orig in _SAVED.pop("kfac", []) + _SAVED.pop("soap", []):
        setattr(owner, attr, orig)
    _TRACES.clear()
