"""The drop-in, end to end: the reference's own optimizers on CUDA through
this library, against the same optimizers on the CPU through the
reference's pure-torch backend.

The reference package is the copy pip-installed under ``baseline/_ref``
(``python -m pip install --no-index --no-build-isolation --target
baseline/_ref <reference checkout>``); ``pytorch_opt_b200.dropin.install``
plugs this library in as its native backend and rewires KFAC. The tests
are skipped when that copy is absent.

* ``test_ops_native_parity_cases``: the cases of the reference's
  ``tests/test_ops_native_parity.py:30-80`` on CUDA tensors, with this
  path's tolerances in place of that file's ``atol`` (which the CPU ATen
  module is held to): Newton–Schulz relative Frobenius error <= 1e-2;
  roots residual <= 1e-4 and relative error <= 1e-4 against the reference;
  factor updates and the two-sided apply relative error <= 1e-4.
* Muon, Shampoo (``root_method="newton"`` and the default eigh route),
  KFAC and EKFAC: a few steps with identical gradients (or identical data)
  on both sides; the parameter change of every matrix is compared with the
  reference's (relative Frobenius error; bounds per optimizer below), and
  the diagnostics that come from the rewired code (``update_rms``,
  ``mean_cond_A/G``) are compared too. SOAP: its factors (the ops call it
  makes), and the size of its update (the update's direction is not
  comparable; see the test).
"""

import os
import sys

import pytest
import torch
from torch import nn

from pytorch_opt_b200 import dropin, native

pytestmark = pytest.mark.gpu

REF_SITE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def po():
    if not os.path.isdir(os.path.join(REF_SITE, "pytorch_opt")):
        pytest.skip("the reference package is not installed under baseline/_ref")
    if REF_SITE not in sys.path:
        sys.path.insert(0, REF_SITE)
    import pytorch_opt
    dropin.install(pytorch_opt)
    yield pytorch_opt
    dropin.uninstall()


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a64 - b64).norm() / b64.norm().clamp_min(1e-300))


def _psd(shape, dtype=torch.float32, seed=11):
    g = torch.Generator().manual_seed(seed)
    B = torch.randn(*shape, generator=g).to(dtype)
    return B @ B.mT + 0.1 * torch.eye(shape[-1], dtype=dtype)


def test_install_routes_cuda_to_native(po, cuda):
    from pytorch_opt import ops
    assert ops._NATIVE is native and ops.native_available()
    A = _psd((5, 5))
    assert torch.equal(ops.inverse_matrix_root(A, 4), ops.reference.inverse_matrix_root(A, 4))  # CPU: reference
    calls = []
    orig = native.newton_schulz_orthogonalize
    native.newton_schulz_orthogonalize = lambda *a: calls.append(1) or orig(*a)
    try:
        ops.newton_schulz_orthogonalize(torch.randn(8, 5, device=cuda))
        ops.set_backend("reference")
        ops.newton_schulz_orthogonalize(torch.randn(8, 5, device=cuda))  # the switch still selects the reference
    finally:
        ops.set_backend("auto")
        native.newton_schulz_orthogonalize = orig
    assert calls == [1]


def test_ops_native_parity_cases(po, cuda):
    """``tests/test_ops_native_parity.py:30-80`` of the reference, on CUDA tensors."""
    from pytorch_opt import ops
    ref = ops.reference
    A, Ab = _psd((6, 6)), _psd((3, 5, 5))
    for p in (1, 2, 4):
        for method in ("eigh", "newton"):
            got = ops.inverse_matrix_root(A.to(cuda), p, damping=1e-6, method=method)
            want = ref.inverse_matrix_root(A, p, damping=1e-6, method=method)
            assert got.is_cuda and _rel(got, want) <= 1e-4, (p, method, _rel(got, want))
    got = ops.inverse_matrix_root(Ab.to(cuda), 4, damping=1e-6)
    assert _rel(got, ref.inverse_matrix_root(Ab, 4, damping=1e-6)) <= 1e-4
    got = ops.inverse_matrix_root(Ab.to(cuda), 4, damping=1e-6, method="newton")
    assert _rel(got, ref.inverse_matrix_root(Ab, 4, damping=1e-6, method="newton")) <= 1e-4
    g = torch.Generator().manual_seed(13)
    for shape in [(8, 5), (5, 8), (4, 6, 9)]:
        G = torch.randn(*shape, generator=g)
        got = ops.newton_schulz_orthogonalize(G.to(cuda))
        assert _rel(got, ref.newton_schulz_orthogonalize(G)) <= 1e-2, shape
    g = torch.Generator().manual_seed(12)
    G1, G2 = (torch.randn(4, 7, generator=g) for _ in range(2))
    for beta2 in (1.0, 0.9):
        Ln, Rn = torch.zeros(4, 4, device=cuda), torch.zeros(7, 7, device=cuda)
        Lr, Rr = torch.zeros(4, 4), torch.zeros(7, 7)
        for G in (G1, G2):
            ops.kron_factor_update_(Ln, Rn, G.to(cuda), beta2=beta2)
            ref.kron_factor_update_(Lr, Rr, G, beta2=beta2)
        assert _rel(Ln, Lr) <= 1e-4 and _rel(Rn, Rr) <= 1e-4
    Lm, G, Rm = torch.randn(4, 4, generator=g), torch.randn(4, 7, generator=g), torch.randn(7, 7, generator=g)
    got = ops.precond_apply_two_sided(Lm.to(cuda), G.to(cuda), Rm.to(cuda))
    assert _rel(got, ref.precond_apply_two_sided(Lm, G, Rm)) <= 1e-4


def _matrix_run(opt_cls, shapes, steps, seed, device, **kw):
    """Run opt_cls over fp32 matrix params with seeded gradients; returns (param changes, optimizer)."""
    g = torch.Generator().manual_seed(seed)
    init = [torch.randn(*s, generator=g) * 0.05 for s in shapes]
    grads = [[torch.randn(*s, generator=g) * 0.02 for s in shapes] for _ in range(steps)]
    params = [nn.Parameter(p.clone().to(device)) for p in init]
    opt = opt_cls(params, **kw)
    for k in range(steps):
        for p, gr in zip(params, grads[k]):
            p.grad = gr.to(device)
        opt.step()
    return [p.detach().cpu() - p0 for p, p0 in zip(params, init)], opt


SHAPES = [(64, 96), (96, 64), (300, 700)]


def test_muon_dropin(po, cuda):
    from pytorch_opt.optim import Muon
    ref, opt_r = _matrix_run(Muon, SHAPES, 3, 1, "cpu", lr=0.02, weight_decay=0.01)
    got, opt_g = _matrix_run(Muon, SHAPES, 3, 1, cuda, lr=0.02, weight_decay=0.01)
    errs = [_rel(a, b) for a, b in zip(got, ref)]
    rms = (opt_g.diagnostics["update_rms"], opt_r.diagnostics["update_rms"])
    print(f"Muon drop-in: parameter-change rel errors {[f'{e:.2e}' for e in errs]}, update_rms {rms}")
    assert max(errs) <= 1e-2
    assert abs(rms[0] - rms[1]) <= 1e-2 * rms[1]


@pytest.mark.parametrize("root_method", ["newton", "auto"])
def test_shampoo_dropin(po, cuda, root_method):
    """Roots are first taken at step 2 (start_step), when every factor has
    full rank. With one gradient, a factor of a non-square matrix is
    singular, and on the reference's eigh route its null-space eigenvalues
    (damping 1e-8 +- fp32 rounding of the factor) decide the result: for
    the 256 x 300 matrix the reference's own CPU factor already has them at
    -2e-8, clamped to 1e-30, so that output is rounding noise in any
    implementation."""
    from pytorch_opt.optim import Shampoo
    kw = dict(lr=0.03, precondition_frequency=1, start_step=2, root_method=root_method, graft="sgd")
    shapes = [(64, 48), (96, 80), (256, 300)]
    ref, _ = _matrix_run(Shampoo, shapes, 4, 2, "cpu", **kw)
    got, _ = _matrix_run(Shampoo, shapes, 4, 2, cuda, **kw)
    errs = [_rel(a, b) for a, b in zip(got, ref)]
    print(f"Shampoo ({root_method}) drop-in: parameter-change rel errors {[f'{e:.2e}' for e in errs]}")
    assert max(errs) <= 1e-3


def test_soap_dropin(po, cuda):
    """SOAP's ops call (``optim/soap.py:95``) is the Kronecker factor update,
    and its rotations into and out of the eigenbases run on the two-sided
    apply kernel (``_soap_update``). Its factors after three steps are
    compared with the reference's. The parameter change is compared with
    eps = 1e-3: with the default eps (1e-8) SOAP's first Adam steps in the
    eigenbasis normalise rotated entries that are zero up to rounding to +-1
    (at step 1 the rotated gradient is diagonal), so even an exactly rounded
    fp32 product moves the default-eps update by ~0.4; with eps = 1e-3 those
    entries stay negligible and the update is well defined."""
    from pytorch_opt.optim import SOAP
    shapes = [(64, 48), (40, 72), (200, 160)]
    calls, moved = [], []
    orig, orig_tr = native.rotate_two_sided, native.soap_transport_
    native.rotate_two_sided = lambda *a, **k: calls.append(1) or orig(*a, **k)
    native.soap_transport_ = lambda *a: moved.append(1) or orig_tr(*a)
    try:
        _, opt_r = _matrix_run(SOAP, shapes, 3, 3, "cpu", lr=3e-3, precondition_frequency=1)
        _, opt_g = _matrix_run(SOAP, shapes, 3, 3, cuda, lr=3e-3, precondition_frequency=1)
        ref, _ = _matrix_run(SOAP, shapes, 3, 3, "cpu", lr=3e-3, precondition_frequency=1, eps=1e-3)
        got, _ = _matrix_run(SOAP, shapes, 3, 3, cuda, lr=3e-3, precondition_frequency=1, eps=1e-3)
    finally:
        native.rotate_two_sided, native.soap_transport_ = orig, orig_tr
    assert len(calls) == 2 * 3 * len(shapes) * 3  # transform(g), transform(m), back(update) per matrix, step, run
    assert len(moved) == 2 * 2 * len(shapes)  # the refreshes of steps 2 and 3 transport the second moment
    ferr = []
    for pg, pr in zip(opt_g.param_groups[0]["params"], opt_r.param_groups[0]["params"]):
        sg, sr = opt_g.state[pg], opt_r.state[pr]
        ferr += [_rel(sg["L"], sr["L"]), _rel(sg["R"], sr["R"])]
    errs = [_rel(a, b) for a, b in zip(got, ref)]
    print(f"SOAP drop-in: factor rel errors {[f'{e:.1e}' for e in ferr]}; eps=1e-3 parameter-change rel errors "
          f"{[f'{e:.2e}' for e in errs]}")
    assert max(ferr) <= 1e-5
    assert max(errs) <= 1e-3


def test_soap_dropin_subspace_refresh(po, cuda):
    """``dropin.install(soap_refresh="subspace")``: after the first refresh
    (fp64 eigh, nothing to start from) every refresh is the warm-started
    subspace iteration (``native.soap_basis`` with the previous basis). The
    factors still equal the reference's (they do not depend on the bases)
    and the bases stay orthonormal to fp32 accuracy. How far the bases and
    the parameters move from the eigh run's is printed, not bounded: on
    these random factors even the top eigenvalues are close together, which
    is where the iteration is an approximation (its convergence on separated
    eigenvalues is asserted in ``test_gpu_soap.py``)."""
    from pytorch_opt.optim import SOAP
    shapes = [(64, 48), (200, 160)]
    warm = []
    orig = native.soap_basis
    native.soap_basis = lambda F, Q_old=None, iters=1, **k: warm.append(Q_old is not None) or orig(F, Q_old, iters, **k)
    dropin.uninstall()
    dropin.install(po, soap_refresh="subspace", soap_iters=2)
    try:
        ref, opt_r = _matrix_run(SOAP, shapes, 3, 3, "cpu", lr=3e-3, precondition_frequency=1, eps=1e-3)
        got, opt_g = _matrix_run(SOAP, shapes, 3, 3, cuda, lr=3e-3, precondition_frequency=1, eps=1e-3)
    finally:
        native.soap_basis = orig
        dropin.uninstall()
        dropin.install(po)
    assert warm == [False, False] * len(shapes) + [True, True] * 2 * len(shapes)
    tops = []
    for pg, pr in zip(opt_g.param_groups[0]["params"], opt_r.param_groups[0]["params"]):
        sg, sr = opt_g.state[pg], opt_r.state[pr]
        assert _rel(sg["L"], sr["L"]) <= 1e-5 and _rel(sg["R"], sr["R"]) <= 1e-5
        for F, Q in ((sg["L"], sg["Q_L"]), (sg["R"], sg["Q_R"])):
            Q64, F64 = Q.double().cpu(), F.double().cpu()
            assert float((Q64.T @ Q64 - torch.eye(Q64.shape[0], dtype=torch.float64)).abs().max()) <= 1e-5
            ev, V = torch.linalg.eigh(F64)
            tops.append(f"{float((Q64[:, -1] @ V[:, -1]).abs()):.3f} (gap {float((ev[-1] - ev[-2]) / ev[-1]):.2f})")
    cos = [float((a.double().flatten() @ b.double().flatten()) / (a.double().norm() * b.double().norm()))
           for a, b in zip(got, ref)]
    assert all(torch.isfinite(a).all() for a in got)
    print(f"SOAP subspace refresh: top-eigenvector |cos| vs eigh {tops}; parameter-change cosine vs the eigh run "
          f"{[f'{c:.3f}' for c in cos]}")


def _mlp():
    torch.manual_seed(5)
    return nn.Sequential(nn.Linear(48, 96), nn.Tanh(), nn.Linear(96, 64), nn.Tanh(), nn.Linear(64, 10))


def _linear():
    torch.manual_seed(5)
    return nn.Sequential(nn.Linear(48, 10))


def _kfac_run(po, opt_name, device, steps=3, model_fn=_mlp):
    from pytorch_opt._testing import mse_half
    import pytorch_opt.optim as optim
    model = model_fn().to(device)
    init = [p.detach().cpu().clone() for p in model.parameters()]
    g = torch.Generator().manual_seed(6)
    X = torch.randn(256, 48, generator=g).to(device)
    y = torch.randn(256, 10, generator=g).to(device)
    opt = getattr(optim, opt_name)(model, lr=0.05, damping=1e-3, inv_every=1)
    for _ in range(steps):
        opt.zero_grad(set_to_none=True)
        mse_half(model(X), y).backward()
        opt.step()
    return [p.detach().cpu() - p0 for p, p0 in zip(model.parameters(), init)], opt


# (optimizer, model, bound on the parameter-change error). EKFAC rescales by
# 1/(s + damping) per element of the factors' eigenbases, which amplifies the
# factors' rounding: perturbing the reference's own CPU factors by 1e-7
# (relative, elementwise) moves its 3-step update by 4e-2 on the 3-layer MLP
# and by 1.5e-4 on one Linear layer (KFAC: 3e-6 and 5e-7). So EKFAC is
# compared on the single layer, with a bound of 5e-3.
KFAC_CASES = [("KFAC", _mlp, 1e-3), ("EKFAC", _linear, 5e-3)]


@pytest.mark.parametrize("opt_name,model_fn,bound", KFAC_CASES, ids=[c[0] for c in KFAC_CASES])
def test_kfac_dropin(po, cuda, opt_name, model_fn, bound):
    ref, opt_r = _kfac_run(po, opt_name, "cpu", model_fn=model_fn)
    got, opt_g = _kfac_run(po, opt_name, cuda, model_fn=model_fn)
    errs = [_rel(a, b) for a, b in zip(got, ref)]
    ca = (opt_g.diagnostics["mean_cond_A"], opt_r.diagnostics["mean_cond_A"])
    cg = (opt_g.diagnostics["mean_cond_G"], opt_r.diagnostics["mean_cond_G"])
    print(f"{opt_name} drop-in: parameter-change rel errors {[f'{e:.2e}' for e in errs]}, mean_cond_A {ca}, "
          f"mean_cond_G {cg}")
    assert max(errs) <= bound
    assert abs(ca[0] - ca[1]) <= 1e-3 * ca[1] and abs(cg[0] - cg[1]) <= 1e-3 * cg[1]
    for name, f in opt_g.tracker.factors.items():  # the factors are the fused kernel's fp32 outputs
        assert f["A"].is_cuda and f["A"].dtype == torch.float32


def test_kfac_traces_from_the_epilogue(po, cuda):
    """kfac_factored_damping reads the traces the SYRK epilogue summed, equal
    to the factors' diagonals, and gives the reference's gammas."""
    from pytorch_opt.curvature.damping import kfac_factored_damping as ref_damping
    from pytorch_opt.optim import kfac as kfac_mod
    _, opt = _kfac_run(po, "KFAC", cuda, steps=2)
    for name, f in opt.tracker.factors.items():
        for key in ("A", "G"):
            t = dropin._trace_of(f[key])
            assert t is not None
            tr = float(t[0][t[1]])
            assert abs(tr - float(f[key].double().diagonal().sum())) <= 1e-5 * abs(tr)
        got = kfac_mod.kfac_factored_damping(f["A"], f["G"], 1e-3)
        want = ref_damping(f["A"].cpu(), f["G"].cpu(), 1e-3)
        assert abs(got[0] - want[0]) <= 1e-5 * want[0] and abs(got[1] - want[1]) <= 1e-5 * want[1]
