"""The drop-in installer on CPU tensors: with this library installed as the
reference's native backend, CPU tensors still take the reference's own
pure-torch path (bit-identical results), the KFAC rewiring falls through to
the reference's code, and ``uninstall`` restores every replaced function.
Skipped when the reference package is not installed under ``baseline/_ref``."""

import os
import sys

import pytest
import torch
from torch import nn

from pytorch_opt_b200 import dropin, native

REF_SITE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def po():
    if not os.path.isdir(os.path.join(REF_SITE, "pytorch_opt")):
        pytest.skip("the reference package is not installed under baseline/_ref")
    if REF_SITE not in sys.path:
        sys.path.insert(0, REF_SITE)
    import pytorch_opt
    return pytorch_opt


def _muon_params(po):
    from pytorch_opt.optim import Muon
    torch.manual_seed(3)
    params = [nn.Parameter(torch.randn(16, 24)), nn.Parameter(torch.randn(24, 16))]
    opt = Muon(params, lr=0.02)
    for _ in range(2):
        for p in params:
            p.grad = torch.randn_like(p) * 0.02
        opt.step()
    return [p.detach().clone() for p in params]


def _kfac_params(po):
    from pytorch_opt._testing import mse_half
    from pytorch_opt.optim import KFAC
    torch.manual_seed(4)
    model = nn.Sequential(nn.Linear(6, 8), nn.Tanh(), nn.Linear(8, 3))
    X, y = torch.randn(32, 6), torch.randn(32, 3)
    opt = KFAC(model, lr=0.1, inv_every=1)
    for _ in range(2):
        opt.zero_grad(set_to_none=True)
        mse_half(model(X), y).backward()
        opt.step()
    return [p.detach().clone() for p in model.parameters()], opt.diagnostics["mean_cond_A"]


def _soap_params(po, **kw):
    from pytorch_opt.optim import SOAP
    torch.manual_seed(6)
    params = [nn.Parameter(torch.randn(12, 20)), nn.Parameter(torch.randn(6, 3, 2, 2)), nn.Parameter(torch.randn(7))]
    opt = SOAP(params, lr=3e-3, precondition_frequency=2, weight_decay=0.01, **kw)
    for _ in range(5):
        for p in params:
            p.grad = torch.randn_like(p) * 0.1
        opt.step()
    return [p.detach().clone() for p in params], opt.diagnostics["stale_steps"], opt.diagnostics["n_adamw_params"]


def test_cpu_tensors_keep_the_reference_path(po):
    from pytorch_opt import ops
    from pytorch_opt.optim import kfac as kfac_mod
    before = {k: getattr(ops, k) for k in ("_NATIVE", "newton_schulz_orthogonalize", "inverse_matrix_root")}
    from pytorch_opt.optim import soap as soap_mod
    k_before = (kfac_mod.kfac_factored_damping, kfac_mod.KFAC.__dict__["_damped_inverse"],
                soap_mod.SOAP.__dict__["_soap_update"])
    muon_ref = _muon_params(po)
    kfac_ref, cond_ref = _kfac_params(po)
    soap_ref = _soap_params(po)
    soap_step = soap_mod.SOAP.__dict__["step"]  # as torch's Optimizer wrapped it at the first construction
    dropin.install(po)
    try:
        assert soap_mod.SOAP.__dict__["step"] is not soap_step  # the restated step (refresh on this library)
        soap_got = _soap_params(po)
        for a, b in zip(soap_got[0], soap_ref[0]):
            assert torch.equal(a, b)
        assert soap_got[1:] == soap_ref[1:]
        assert ops._NATIVE is native and ops.newton_schulz_orthogonalize is not before["newton_schulz_orthogonalize"]
        A = torch.randn(6, 6, dtype=torch.float64)
        A = A @ A.T + torch.eye(6, dtype=torch.float64)
        assert torch.equal(ops.inverse_matrix_root(A, 4, method="newton"),
                           ops.reference.inverse_matrix_root(A, 4, method="newton"))
        for a, b in zip(_muon_params(po), muon_ref):
            assert torch.equal(a, b)
        kfac_got, cond_got = _kfac_params(po)
        for a, b in zip(kfac_got, kfac_ref):
            assert torch.equal(a, b)
        assert cond_got == cond_ref
    finally:
        dropin.uninstall()
    for k, v in before.items():
        assert getattr(ops, k) is v
    assert (kfac_mod.kfac_factored_damping, kfac_mod.KFAC.__dict__["_damped_inverse"],
            soap_mod.SOAP.__dict__["_soap_update"]) == k_before
    assert soap_mod.SOAP.__dict__["step"] is soap_step
