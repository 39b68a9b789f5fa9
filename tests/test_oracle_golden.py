"""The numpy oracle against golden vectors produced by the reference itself.

``tests/golden/*.npz`` were written by ``tests/golden/make_golden.py`` from
kavinravi/pytorch-opt's own ``ops.reference``, ``KronTracker``,
``kfac_factored_damping``, ``KFAC._damped_inverse`` and ``Muon`` on seeded
inputs. Passing here pins ``oracle/ops_np.py`` before it is trusted as the
checker of the GPU kernels.
"""

import os

import numpy as np
import pytest

from oracle import ops_np as O
from tests.conftest import GOLDEN_DIR


def _load(name):
    return np.load(os.path.join(GOLDEN_DIR, name))


def _rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def test_newton_schulz_golden():
    z = _load("ns.npz")
    for i in range(int(z["ncases"])):
        x, want, (steps, dt) = z[f"case{i}_in"], z[f"case{i}_out"], z[f"case{i}_meta"]
        got = O.newton_schulz(x, int(steps), out_bf16=(dt == 1))
        tol = {0: 1e-5, 1: 2e-3, 3: 1e-12}[int(dt)]
        assert _rel(got, want) < tol, (i, _rel(got, want))


def test_inverse_root_golden():
    z = _load("roots.npz")
    for i in range(int(z["ncases"])):
        A, want, (p, damping, m) = z[f"case{i}_in"], z[f"case{i}_out"], z[f"case{i}_meta"]
        method = ("auto", "eigh", "newton")[int(m)]
        got = O.inverse_matrix_root(A, int(p), damping=float(damping), method=method)
        tol = 1e-10 if A.dtype == np.float64 else 1e-6
        assert got.dtype == A.dtype
        assert _rel(got, want) < tol, (i, method, _rel(got, want))


def test_inverse_root_argument_errors():
    A = np.eye(3)
    with pytest.raises(ValueError, match="positive integer"):
        O.inverse_matrix_root(A, 0)
    with pytest.raises(ValueError, match="method"):
        O.inverse_matrix_root(A, 2, method="qr")


def test_kron_factor_update_golden():
    z = _load("kron.npz")
    for i in range(int(z["ncases"])):
        G1, G2 = z[f"case{i}_G1"], z[f"case{i}_G2"]
        m, n = G1.shape
        for beta in (1.0, 0.9):
            L, R = np.zeros((m, m), np.float32), np.zeros((n, n), np.float32)
            L, R = O.kron_factor_update(L, R, G1, beta)
            L, R = O.kron_factor_update(L, R, G2, beta)
            assert _rel(L, z[f"case{i}_L_{beta}"]) < 1e-6
            assert _rel(R, z[f"case{i}_R_{beta}"]) < 1e-6
    with pytest.raises(ValueError, match="2D"):
        O.kron_factor_update(np.zeros((2, 2)), np.zeros((2, 2)), np.zeros((2, 2, 2)))


def test_precond_golden():
    z = _load("precond.npz")
    for i in range(int(z["ncases"])):
        got = O.precond_apply(z[f"case{i}_L"], z[f"case{i}_G"], z[f"case{i}_R"])
        assert _rel(got, z[f"case{i}_out"]) < 1e-6


def test_kfac_factors_damping_inverse_golden():
    z = _load("kfac.npz")
    for i in range(int(z["ncases"])):
        bias, ema = z[f"case{i}_meta"]
        ema = None if ema < 0 else float(ema)
        A = G = None
        for step in range(3):
            Ab, Gb = O.kfac_batch_factors_linear(z[f"case{i}_a{step}"], z[f"case{i}_g{step}"], bool(bias))
            A = O.kfac_update(A, Ab, ema, step)
            G = O.kfac_update(G, Gb, ema, step)
        assert _rel(A, z[f"case{i}_A"]) < 1e-6
        assert _rel(G, z[f"case{i}_G"]) < 1e-6
        ga, gg = O.kfac_factored_damping(z[f"case{i}_A"], z[f"case{i}_G"], 1e-3)
        np.testing.assert_allclose([ga, gg], z[f"case{i}_gammas"], rtol=1e-6)  # fp32 traces
        iA, cA = O.kfac_damped_inverse(z[f"case{i}_A"], ga)
        iG, cG = O.kfac_damped_inverse(z[f"case{i}_G"], gg)
        assert _rel(iA, z[f"case{i}_iA"]) < 1e-6 and _rel(iG, z[f"case{i}_iG"]) < 1e-6
        np.testing.assert_allclose([cA, cG], z[f"case{i}_conds"], rtol=1e-6)


def test_muon_golden():
    z = _load("muon.npz")
    lr, mom, nest, steps, wd = z["hparams"]
    for k in range(int(z["nparams"])):
        p, buf = z[f"p{k}_init"], np.zeros_like(z[f"p{k}_init"])
        for s in range(2):
            p, buf, _, _ = O.muon_matrix_step(p, z[f"p{k}_grad{s}"], buf, lr=float(lr), momentum=float(mom),
                                              nesterov=bool(nest), ns_steps=int(steps), weight_decay=float(wd))
        # Momentum never passes through a matrix product: bit-exact.
        np.testing.assert_array_equal(buf, z[f"p{k}_buf"])
        # The update goes through fp32 products whose summation order differs
        # from torch's; after bf16 rounding a few elements may differ by an ulp.
        dp_got, dp_want = p - z[f"p{k}_init"], z[f"p{k}_final"] - z[f"p{k}_init"]
        assert _rel(dp_got, dp_want) < 2e-2, _rel(dp_got, dp_want)
        assert np.mean(p != z[f"p{k}_final"]) < 0.05


def test_bf16_round_matches_torch():
    import torch
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 7.3
    x[:4] = [0.0, -0.0, 1e-40, 3.0e38]
    want = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(O.bf16_round(x), want)


def test_ekfac_oracle_matches_reference_golden():
    z = np.load(os.path.join(GOLDEN_DIR, "ekfac.npz"))
    for i in range(int(z["ncases"])):
        decay, lam = (float(v) for v in z[f"case{i}_hp"])
        QG, QA = z[f"case{i}_QG"], z[f"case{i}_QA"]
        o1, s1 = O.ekfac_precondition(QG, QA, z[f"case{i}_V1"], None, decay, lam)
        o2, s2 = O.ekfac_precondition(QG, QA, z[f"case{i}_V2"], s1, decay, lam)
        for got, key in ((o1, "out1"), (s1, "s1"), (o2, "out2"), (s2, "s2")):
            want = z[f"case{i}_{key}"]
            assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-5, (i, key)



def test_soap_refresh_oracle_matches_reference_golden():
    """The reference's SOAP refreshed its bases every step; from the state
    before and after each refresh: the oracle's bases are eigenbases of the
    new factors matching the reference's up to column signs, and the
    oracle's transport, followed by the step's second-moment EMA, gives the
    reference's second moment."""
    z = np.load(os.path.join(GOLDEN_DIR, "soap.npz"))
    b2, _ = (float(v) for v in z["hp"])
    for k in range(1, int(z["nsteps"])):
        L, R = z[f"step{k}_L"], z[f"step{k}_R"]
        ql, qr = O.soap_bases(L, R)
        for mine, ref in ((ql, z[f"step{k}_QL"]), (qr, z[f"step{k}_QR"])):
            cos = np.abs(np.sum(mine.astype(np.float64) * ref, axis=0))
            assert cos.min() >= 1 - 1e-4, (k, cos.min())
        ql, qr = z[f"step{k}_QL"].astype(np.float64), z[f"step{k}_QR"].astype(np.float64)
        carried = O.soap_transport(z[f"step{k - 1}_V"], z[f"step{k - 1}_QL"], ql, z[f"step{k - 1}_QR"], qr)
        g_rot = ql.T @ z[f"step{k}_grad"].astype(np.float64) @ qr
        want = z[f"step{k}_V"]
        got = b2 * carried + (1 - b2) * g_rot * g_rot
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-5, k


# --------------------------------------------------- torch full-size checker
# oracle/ops_torch.py evaluates the same algorithms with torch (on the GPU in
# the full-size parity tests); here it is pinned on the CPU to the same
# golden vectors as the numpy restatement.

def test_torch_checker_newton_schulz_golden():
    import torch
    from oracle import ops_torch as T
    z = _load("ns.npz")
    for i in range(int(z["ncases"])):
        x, want, (steps, dt) = z[f"case{i}_in"], z[f"case{i}_out"], z[f"case{i}_meta"]
        G = torch.from_numpy(x).to({0: torch.float32, 1: torch.bfloat16, 3: torch.float64}[int(dt)])
        got = T.newton_schulz(G, int(steps)).double().numpy()
        tol = {0: 1e-5, 1: 2e-3, 3: 1e-12}[int(dt)]
        assert _rel(got, want) < tol, (i, _rel(got, want))


def test_torch_checker_newton_roots_golden():
    import torch
    from oracle import ops_torch as T
    z = _load("roots.npz")
    for i in range(int(z["ncases"])):
        A, want, (p, damping, m) = z[f"case{i}_in"], z[f"case{i}_out"], z[f"case{i}_meta"]
        if ("auto", "eigh", "newton")[int(m)] != "newton" or A.ndim != 2:
            continue
        X, its = T.inverse_root_newton(torch.from_numpy(A), int(p), float(damping))
        _, its_np = O.coupled_newton(0.5 * (A + A.T).astype(np.float64) + float(damping) * np.eye(A.shape[0]), int(p))
        assert its == its_np
        assert _rel(X.numpy().astype(A.dtype), want) < (1e-10 if A.dtype == np.float64 else 1e-6), i


def test_torch_checker_kfac_golden():
    import torch
    from oracle import ops_torch as T
    z = _load("kfac.npz")
    for i in range(int(z["ncases"])):
        bias, ema = z[f"case{i}_meta"]
        if ema < 0:
            continue
        FA = FG = None
        for step in range(3):
            a = torch.from_numpy(z[f"case{i}_a{step}"])
            g = torch.from_numpy(z[f"case{i}_g{step}"])
            n = a.shape[0]
            if bias:
                a = torch.cat([a, torch.ones(n, 1)], dim=1)
            FA = T.kfac_update(FA, T.kron_batch_factor(a, 1.0 / n), float(ema))
            FG = T.kfac_update(FG, T.kron_batch_factor(g, float(n)), float(ema))
        assert _rel(FA.numpy(), z[f"case{i}_A"]) < 1e-6 and _rel(FG.numpy(), z[f"case{i}_G"]) < 1e-6
        ga, gg = z[f"case{i}_gammas"]
        iA, cA = T.damped_inverse(torch.from_numpy(z[f"case{i}_A"]), float(ga))
        iG, cG = T.damped_inverse(torch.from_numpy(z[f"case{i}_G"]), float(gg))
        assert _rel(iA.numpy(), z[f"case{i}_iA"]) < 1e-6 and _rel(iG.numpy(), z[f"case{i}_iG"]) < 1e-6
        np.testing.assert_allclose([cA, cG], z[f"case{i}_conds"], rtol=1e-10)


def test_full_size_fixture_is_complete():
    """The full-size fixture holds what the GPU tests read, and the reference's
    iteration counts on config 3 (d = 1024 / 2048 / 4096)."""
    z = _load("full_size.npz")
    for i in range(4):
        assert z[f"ns{i}_sketch"].shape == (32, 32)
    assert [int(z[f"root{d}_iters"]) for d in (1024, 2048, 4096)] == [10, 11, 11]
    assert z["kfac_iA_sketch"].shape == (32, 32) and z["kfac_conds"].shape == (2,)
