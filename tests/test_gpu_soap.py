"""SOAP's basis refresh on the device (``pytorch_opt/optim/soap.py:96-110``).

* ``soap_transport_`` (``po_soap_transport``) against the oracle's fp64
  restatement of the reference's transport, fp32 (split-tf32 products,
  relative Frobenius error <= 1e-5) and bf16 (<= 2e-2); under a permutation
  with sign flips of the basis, the case the reference's docstring calls
  exact, it permutes V up to the split-tf32 representation of V (hi + lo
  keeps 22 of fp32's 24 significant bits: every element within 2^-20
  relative).
* ``soap_basis`` (warm-started subspace iteration): a basis that already
  diagonalises the factor is a fixed point (up to order and signs, which it
  restores to eigh's ascending order); on a factor with a few well-separated
  eigenvalues above a bulk, perturbed from the previous one, the separated
  eigenvectors converge to the fp64 eigh's (|cos| >= 0.9999) and the second
  moment transported with these bases matches the one transported with
  eigh's bases on those directions (<= 1e-3). Inside the bulk, where
  neighbouring eigenvalues differ by less than the perturbation, the
  iteration does not resolve single eigenvectors; that is the approximation
  the method makes, and it is not asserted.
"""

import numpy as np
import pytest
import torch

from oracle import ops_np as O
from pytorch_opt_b200 import native

pytestmark = pytest.mark.gpu


def _orth(d, g):
    return torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64))[0]


def _rel(a, b) -> float:
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("m,n", [(64, 48), (200, 160), (1024, 512)])
def test_soap_transport_matches_oracle(cuda, m, n):
    g = torch.Generator().manual_seed(m + n)
    qlo, qro = _orth(m, g), _orth(n, g)
    # new bases: the old ones rotated by a moderate random rotation
    qln = torch.linalg.qr(qlo + 0.3 * torch.randn(m, m, generator=g, dtype=torch.float64))[0]
    qrn = torch.linalg.qr(qro + 0.3 * torch.randn(n, n, generator=g, dtype=torch.float64))[0]
    V = torch.rand(m, n, generator=g, dtype=torch.float64) ** 2
    for dt, tol in ((torch.float32, 1e-5), (torch.bfloat16, 2e-2)):
        ts = [t.to(dt) for t in (V, qlo, qln, qro, qrn)]
        want = O.soap_transport(*[t.float().numpy() for t in ts])
        got = native.soap_transport_(ts[0].to(cuda), *[t.to(cuda) for t in ts[1:]])
        err = _rel(got.float().cpu().numpy(), want)
        print(f"soap_transport {m}x{n} {dt}: rel err {err:.2e}")
        assert err <= tol


def test_soap_transport_is_exact_under_permutation_and_signs(cuda):
    m, n = 96, 80
    g = torch.Generator().manual_seed(3)
    qlo, qro = _orth(m, g).float(), _orth(n, g).float()
    pl, pr = torch.randperm(m, generator=g), torch.randperm(n, generator=g)
    sl = torch.where(torch.rand(m, generator=g) < 0.5, -1.0, 1.0)
    sr = torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0)
    qln, qrn = qlo[:, pl] * sl, qro[:, pr] * sr
    V = torch.rand(m, n, generator=g)
    # C_L = Q_L_old^T Q_L_new is the signed permutation only up to rounding of
    # the orthogonality of Q_L_old; build it from an exactly orthogonal basis.
    eye_l, eye_r = torch.eye(m), torch.eye(n)
    got = native.soap_transport_(V.to(cuda), eye_l.to(cuda), (eye_l[:, pl] * sl).to(cuda), eye_r.to(cuda),
                                 (eye_r[:, pr] * sr).to(cuda)).cpu()
    want = V[pl][:, pr]
    assert float(((got - want).abs() / want.abs()).max()) <= 2.0 ** -20
    # and with a rounded orthogonal basis it is the permutation to fp32 accuracy
    got = native.soap_transport_(V.to(cuda), qlo.to(cuda), qln.to(cuda), qro.to(cuda), qrn.to(cuda)).cpu()
    assert _rel(got.numpy(), V[pl][:, pr].numpy()) <= 1e-5


def _spiked(d, g, spikes=8):
    """Factor with `spikes` eigenvalues 2x apart above a bulk in [1e-3, 1e-2]."""
    Q = _orth(d, g)
    lam = torch.cat([torch.logspace(-3, -2, d - spikes, dtype=torch.float64),
                     0.1 * 2.0 ** torch.arange(spikes, dtype=torch.float64)])
    return Q, lam


def test_soap_basis_fixed_point(cuda):
    d = 256
    g = torch.Generator().manual_seed(5)
    Q, lam = _spiked(d, g)
    lam = torch.logspace(-2, 0, d, dtype=torch.float64)  # every eigenvalue distinct
    F = (Q * lam) @ Q.T
    perm = torch.randperm(d, generator=g)
    signs = torch.where(torch.rand(d, generator=g) < 0.5, -1.0, 1.0).double()
    Qs = native.soap_basis(F.float().to(cuda), (Q[:, perm] * signs).float().to(cuda), iters=2).double().cpu()
    cos = (Qs * Q).sum(0).abs()  # Q's columns are in ascending eigenvalue order
    print(f"soap_basis fixed point: min |cos| {float(cos.min()):.7f}")
    assert float(cos.min()) >= 1 - 1e-4
    assert float((Qs.T @ Qs - torch.eye(d, dtype=torch.float64)).abs().max()) <= 1e-5


@pytest.mark.parametrize("d", [256, 1024])
def test_soap_basis_warm_start_separated_directions(cuda, d):
    g = torch.Generator().manual_seed(d)
    Q, lam = _spiked(d, g)
    F0 = (Q * lam) @ Q.T
    N = torch.randn(d, d, generator=g, dtype=torch.float64)
    F1 = F0 + 1e-3 * (N + N.T) / d ** 0.5
    Qold = torch.linalg.eigh(F0)[1]
    ev, Qe = torch.linalg.eigh(F1)
    Qs = native.soap_basis(F1.float().to(cuda), Qold.float().to(cuda), iters=2).double().cpu()
    top = slice(d - 8, d)
    cos_old = (Qold[:, top] * Qe[:, top]).sum(0).abs()
    cos = (Qs[:, top] * Qe[:, top]).sum(0).abs()
    orth = float((Qs.T @ Qs - torch.eye(d, dtype=torch.float64)).abs().max())
    print(f"soap_basis d={d}: separated |cos| warm start {float(cos_old.min()):.6f} -> {float(cos.min()):.7f}; "
          f"orthogonality {orth:.1e}")
    assert float(cos.min()) >= 0.9999 and float(cos.min()) >= float(cos_old.min())
    assert orth <= 1e-5
    # the rotated second moment carried into these bases vs into eigh's, on the separated directions
    m2 = 64
    Qr = _orth(m2, g)
    V = torch.rand(d, m2, generator=g, dtype=torch.float64) ** 2
    ref = O.soap_transport(V.numpy(), Qold.numpy(), Qe.numpy(), Qr.numpy(), Qr.numpy())
    got = native.soap_transport_(V.float().to(cuda), Qold.float().to(cuda), Qs.float().to(cuda),
                                 Qr.float().to(cuda), Qr.float().to(cuda)).double().cpu().numpy()
    err = _rel(got[top], ref[top])
    print(f"  transported moments on the separated directions: rel err {err:.1e}")
    assert err <= 1e-3
