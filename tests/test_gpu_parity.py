"""GPU parity of the sm_100a kernels against the reference (golden vectors)
and the numpy oracle, through the C ABI (via ``pytorch_opt_b200.native``).

Tolerances (stated by the task for this path):
* Newton–Schulz (bf16/tf32 tensor-core products): relative Frobenius error
  <= 1e-2 against the reference's fp32 result on the same input;
* inverse roots: residual ||X^p (A + eps I) - I||_F / sqrt(d) <= 1e-4 (fp64
  evaluation of the returned X), plus the same iteration count as the
  reference's fp64 loop;
* factor updates: relative Frobenius error <= 1e-4.
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import ops_np as O
from pytorch_opt_b200 import _lib, native, ops
from pytorch_opt_b200.muon import GroupedMuon, MuonGroup
from tests.conftest import GOLDEN_DIR

pytestmark = pytest.mark.gpu

NS_TOL = 1e-2
ROOT_TOL = 1e-4
FACTOR_TOL = 1e-4
TORCH_DT = {0: torch.float32, 1: torch.bfloat16, 3: torch.float64}


def _rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float64 if t.dtype == torch.float64 else torch.float32).numpy()


@pytest.fixture(autouse=True)
def _device_error_stays_clear(cuda):
    yield
    assert _lib.device_error(reset=True) == 0


def test_native_library_is_the_in_tree_build(cuda):
    lib = _lib.load()
    assert os.path.dirname(_lib.LIB_PATH).endswith("pytorch_opt_b200")
    assert b"sm_100a" in lib.po_version()
    assert torch.cuda.get_device_capability(cuda)[0] == 10


@pytest.mark.parametrize("sleeping", [0, 1])
def test_bounded_wait_gives_up_and_reports(cuda, sleeping):
    """A kernel wait on a barrier nothing arms ends after its limit (20 ms
    here instead of 5 s): the kernel returns, po_device_error() reports code
    5 once, and the context keeps working (a product runs afterwards)."""
    import time
    lib = _lib.load()
    assert _lib.device_error(reset=True) == 0
    t0 = time.perf_counter()
    _lib.check(lib.po_selftest_wait_timeout(20_000_000, sleeping, _lib.stream_ptr(cuda)), "selftest")
    code = _lib.device_error(reset=True)
    took = time.perf_counter() - t0
    assert code == 5, code
    assert took < 5.0, took
    assert _lib.device_error(reset=True) == 0  # reset clears it
    G = torch.randn(64, 96, device=cuda)
    assert _rel(_np(ops.newton_schulz_orthogonalize(G)), O.newton_schulz(_np(G))) <= NS_TOL


# ---------------------------------------------------------------- Newton–Schulz

def test_ns_golden(cuda):
    z = np.load(os.path.join(GOLDEN_DIR, "ns.npz"))
    for i in range(int(z["ncases"])):
        x, want, (steps, dt) = z[f"case{i}_in"], z[f"case{i}_out"], z[f"case{i}_meta"]
        G = torch.from_numpy(x).to(cuda, TORCH_DT[int(dt)])
        got = native.newton_schulz_orthogonalize(G, int(steps), 3.4445, -4.7750, 2.0315, 1e-7)
        assert got.dtype == G.dtype and got.shape == G.shape
        assert _rel(_np(got), want) <= NS_TOL, (i, _rel(_np(got), want))


@pytest.mark.parametrize("shape,dtype,scale", [
    ((768, 3072), torch.float32, 1.0),      # config 1
    ((768, 2304), torch.bfloat16, 0.02),    # GPT-2 qkv
    ((3072, 768), torch.bfloat16, 0.02),    # GPT-2 proj (tall: transposed path)
    ((768, 768), torch.bfloat16, 0.02),     # GPT-2 attn-out
    ((1024, 4096), torch.bfloat16, 0.02),   # Llama k/v
    ((3, 200, 96), torch.float32, 1.0),     # batched, tall, small (split schedule)
    ((300, 700), torch.float32, 1.0),       # tf32 schedule
    ((129, 257), torch.float32, 1.0),       # ragged tiles
    ((1, 7), torch.float32, 1.0), ((7, 1), torch.float32, 1.0), ((1, 1), torch.float32, 1.0),
    ((64, 100), torch.float16, 1.0), ((40, 24), torch.float64, 1.0),
])
def test_ns_vs_oracle(cuda, shape, dtype, scale):
    g = torch.Generator().manual_seed(sum(shape))
    Gc = (torch.randn(*shape, generator=g) * scale).to(dtype)
    want = O.newton_schulz(_np(Gc).astype(np.float64 if dtype == torch.float64 else np.float32), 5,
                           out_bf16=(dtype == torch.bfloat16))
    got = ops.newton_schulz_orthogonalize(Gc.to(cuda))
    assert got.dtype == dtype and got.shape == Gc.shape
    assert _rel(_np(got), want) <= NS_TOL


@pytest.mark.parametrize("shape,steps", [((512, 1536), 5), ((1536, 512), 5), ((320, 700), 2), ((700, 320), 3),
                                         ((2, 384, 1024), 4), ((1024, 384), 6)])
def test_ns_grouped_steps(cuda, shape, steps, monkeypatch):
    """Matrices with n >= 2m (m >= 256) run their steps in groups of up to
    three (one tall Gram and one tall update per group, the steps in between
    as m x m products): within the NS tolerance of the oracle, and of the
    one-step-at-a-time schedule (PO_NS_GROUP=0) for 2 .. 6 steps."""
    g = torch.Generator().manual_seed(sum(shape) + steps)
    Gc = (torch.randn(*shape, generator=g) * 0.02).bfloat16()
    want = O.newton_schulz(_np(Gc), steps, out_bf16=True)
    G = Gc.to(cuda)
    got = native.newton_schulz_orthogonalize(G, steps, 3.4445, -4.7750, 2.0315, 1e-7)
    monkeypatch.setenv("PO_NS_GROUP", "0")
    one = native.newton_schulz_orthogonalize(G, steps, 3.4445, -4.7750, 2.0315, 1e-7)
    monkeypatch.delenv("PO_NS_GROUP")
    e_group, e_one, e_between = _rel(_np(got), want), _rel(_np(one), want), _rel(_np(got), _np(one))
    print(f"NS {tuple(shape)} x{steps}: grouped {e_group:.2e}, one step at a time {e_one:.2e}, between {e_between:.2e}")
    assert e_group <= NS_TOL and e_one <= NS_TOL and e_between <= NS_TOL


def test_ns_noncontiguous_and_zero_and_steps0(cuda):
    G = torch.randn(96, 64, device=cuda).T  # non-contiguous view
    want = O.newton_schulz(_np(G.contiguous()))
    assert _rel(_np(ops.newton_schulz_orthogonalize(G)), want) <= NS_TOL
    Z = torch.zeros(32, 48, device=cuda)
    assert torch.count_nonzero(ops.newton_schulz_orthogonalize(Z)) == 0
    X = torch.randn(16, 24, device=cuda)
    want0 = O.newton_schulz(_np(X), 0)
    assert _rel(_np(ops.newton_schulz_orthogonalize(X, steps=0)), want0) < 1e-6
    E = torch.empty(0, 5, device=cuda)
    assert ops.newton_schulz_orthogonalize(E).shape == (0, 5)


def test_ns_full_size_llama_gate_band(cuda):
    """Full Llama-3-8B gate shape: size-independent property (singular values in NS5's band)."""
    g = torch.Generator(device=cuda).manual_seed(7)
    G = (torch.randn(14336, 4096, device=cuda, generator=g) * 0.02).bfloat16()
    Ob = ops.newton_schulz_orthogonalize(G)
    s = torch.linalg.svdvals(Ob.float())
    assert float(s.min()) > 0.55 and float(s.max()) < 1.25
    # and a sampled oracle check on a slice of the same distribution
    sub = G[:1024, :512].contiguous()
    assert _rel(_np(ops.newton_schulz_orthogonalize(sub)), O.newton_schulz(_np(sub), 5, out_bf16=True)) <= NS_TOL


# ----------------------------------------------------------------------- roots

def _shampoo_factor(d, seed):
    g = torch.Generator().manual_seed(seed)
    G = torch.randn(d, 2 * d, generator=g)
    return G @ G.T / (2 * d) + 1e-6 * torch.eye(d)


def test_root_golden(cuda):
    z = np.load(os.path.join(GOLDEN_DIR, "roots.npz"))
    for i in range(int(z["ncases"])):
        A, want, (p, damping, m) = z[f"case{i}_in"], z[f"case{i}_out"], z[f"case{i}_meta"]
        method = ("auto", "eigh", "newton")[int(m)]
        got = ops.inverse_matrix_root(torch.from_numpy(A).to(cuda), int(p), damping=float(damping), method=method)
        assert got.dtype == torch.from_numpy(A).dtype
        assert O.root_residual(_np(got), A, int(p), float(damping)) <= ROOT_TOL, i
        assert _rel(_np(got), want) <= 1e-4, (i, method, _rel(_np(got), want))


@pytest.mark.parametrize("d,p", [(256, 4), (512, 4), (1024, 4), (300, 2), (257, 1), (1000, 3)])
def test_root_newton_vs_oracle_iterations(cuda, d, p):
    L = _shampoo_factor(d, d * 100)
    Ld = _np(L).astype(np.float64)
    want, its = O.coupled_newton(0.5 * (Ld + Ld.T) + 1e-8 * np.eye(d), p)  # reference.py:58-62 then :17-40
    it_dev = torch.zeros(1, dtype=torch.int32, device=cuda)
    A = L.to(cuda)
    lib = _lib.load()
    out = torch.empty_like(A)
    nbytes = lib.po_root_workspace_bytes(1, d, p)
    ws = _lib.workspace(nbytes, cuda)
    _lib.check(lib.po_inverse_root(A.data_ptr(), 0, 1, d, d, d * d, out.data_ptr(), d, d * d, p, 1e-8, 100, 1e-10,
                                   it_dev.data_ptr(), ws.data_ptr(), nbytes, _lib.stream_ptr(cuda)), "root")
    assert int(it_dev.item()) == its  # same stopping step as the fp64 reference loop
    assert O.root_residual(_np(out), _np(L), p, 1e-8) <= ROOT_TOL
    assert _rel(_np(out), 0.5 * (want + want.T)) <= 1e-4


def test_root_full_size_shampoo_4096(cuda):
    """Config 3's largest factors, batched: residual bound on every item."""
    g = torch.Generator(device=cuda).manual_seed(4096)
    Gs = torch.randn(2, 4096, 8192, device=cuda, generator=g)
    Ls = Gs @ Gs.mT / 8192 + 1e-6 * torch.eye(4096, device=cuda)
    del Gs
    X = native.inverse_matrix_root(Ls, 4, 1e-8, "newton", True, 100, 1e-10)
    for i in range(2):
        Xd = X[i].double()
        R = torch.linalg.matrix_power(Xd, 4) @ (Ls[i].double() + 1e-8 * torch.eye(4096, device=cuda,
                                                                               dtype=torch.float64))
        R -= torch.eye(4096, device=cuda, dtype=torch.float64)
        assert float(R.norm() / 64.0) <= ROOT_TOL


def test_root_batched_mixed_conditioning(cuda):
    """Items of one batch converge after different step counts; each matches its own reference."""
    mats = [_shampoo_factor(200, 1), _shampoo_factor(200, 2) * 50.0, torch.eye(200) * 3.0]
    A = torch.stack(mats)
    X = ops.inverse_matrix_root(A.to(cuda), 4, damping=1e-6, method="newton")
    for i, M in enumerate(mats):
        ref = O.inverse_matrix_root(_np(M), 4, 1e-6, "newton")
        assert O.root_residual(_np(X[i]), _np(M), 4, 1e-6) <= ROOT_TOL
        assert _rel(_np(X[i]), ref) <= 1e-4


def test_root_dtypes_and_eigh_route(cuda):
    L = _shampoo_factor(64, 3)
    for dt in (torch.float32, torch.float64):
        X = ops.inverse_matrix_root(L.to(cuda, dt), 4, damping=1e-6, method="newton")
        assert X.dtype == dt
        assert O.root_residual(_np(X), _np(L.to(dt)), 4, 1e-6) <= ROOT_TOL
    # bf16 in, bf16 out: the root of the bf16-valued input, rounded once to bf16.
    Lb = L.to(torch.bfloat16)
    Xb = ops.inverse_matrix_root(Lb.to(cuda), 4, damping=1e-6, method="newton")
    assert Xb.dtype == torch.bfloat16
    want = O.inverse_matrix_root(_np(Lb).astype(np.float64), 4, 1e-6, "newton")
    assert _rel(_np(Xb), want) <= 2.0 ** -8
    Xe = ops.inverse_matrix_root(L.to(cuda), 4, damping=1e-6, method="eigh")
    assert O.root_residual(_np(Xe), _np(L), 4, 1e-6) <= 1e-6


# ------------------------------------------------------------- factor updates

def test_kron_golden(cuda):
    z = np.load(os.path.join(GOLDEN_DIR, "kron.npz"))
    for i in range(int(z["ncases"])):
        G1, G2 = (torch.from_numpy(z[f"case{i}_{k}"]).to(cuda) for k in ("G1", "G2"))
        m, n = G1.shape
        for beta in (1.0, 0.9):
            L, R = torch.zeros(m, m, device=cuda), torch.zeros(n, n, device=cuda)
            ops.kron_factor_update_(L, R, G1, beta2=beta)
            out = ops.kron_factor_update_(L, R, G2, beta2=beta)
            assert out[0] is L and out[1] is R
            assert _rel(_np(L), z[f"case{i}_L_{beta}"]) <= FACTOR_TOL
            assert _rel(_np(R), z[f"case{i}_R_{beta}"]) <= FACTOR_TOL


@pytest.mark.parametrize("m,n,dt,beta", [(1024, 768, torch.float32, 0.999), (768, 3072, torch.bfloat16, 0.95),
                                         (33, 17, torch.float32, 1.0), (1, 5, torch.float32, 0.9)])
def test_kron_vs_oracle(cuda, m, n, dt, beta):
    g = torch.Generator().manual_seed(m * n)
    L0 = _shampoo_factor(m, 1)
    R0 = _shampoo_factor(n, 2)
    G = torch.randn(m, n, generator=g).to(dt)
    L, R = L0.to(cuda), R0.to(cuda)
    ops.kron_factor_update_(L, R, G.to(cuda), beta2=beta)
    Lw, Rw = O.kron_factor_update(_np(L0).astype(np.float64), _np(R0).astype(np.float64), _np(G).astype(np.float64),
                                  beta)
    assert _rel(_np(L), Lw) <= FACTOR_TOL and _rel(_np(R), Rw) <= FACTOR_TOL


@pytest.mark.parametrize("rows,d,dt", [(4096, 2048, torch.bfloat16), (1000, 300, torch.float32),
                                       (77, 33, torch.bfloat16), (8192, 1024, torch.float32)])
def test_kfac_syrk_ema_vs_oracle(cuda, rows, d, dt):
    """KronTracker semantics: first call clones a^T a / n, then EMA with beta = 0.95."""
    g = torch.Generator().manual_seed(rows + d)
    a1, a2 = (torch.randn(rows, d, generator=g).to(dt) for _ in range(2))
    F = torch.empty(d, d, device=cuda)
    native.kron_syrk_ema_(F, a1.to(cuda), 1.0 / rows, 0.95, True)
    native.kron_syrk_ema_(F, a2.to(cuda), 1.0 / rows, 0.95, False)
    A1 = _np(a1).astype(np.float64)
    A2 = _np(a2).astype(np.float64)
    want = O.kfac_update(O.kfac_update(None, A1.T @ A1 / rows, 0.95), A2.T @ A2 / rows, 0.95)
    assert _rel(_np(F), want) <= FACTOR_TOL


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_band_split_factor_update_one_rank(cuda, dt):
    """The band-split factor update (one rank: one band product + mirror)
    against the fused SYRK-EMA kernel and the oracle (first call and EMA)."""
    from pytorch_opt_b200.dist import sharded_syrk_ema_
    g = torch.Generator().manual_seed(21)
    rows, d = 2048, 700
    X1 = torch.randn(rows, d, generator=g).to(dt)
    X2 = torch.randn(rows, d, generator=g).to(dt)
    Fa = torch.empty(d, d, device=cuda)
    Fb = torch.empty(d, d, device=cuda)
    for X, first in ((X1, True), (X2, False)):
        sharded_syrk_ema_(Fa, X.to(cuda), 1.0 / rows, 0.95, first)
        native.kron_syrk_ema_(Fb, X.to(cuda), 1.0 / rows, 0.95, first)
    assert _rel(_np(Fa), _np(Fb).astype(np.float64)) <= 1e-5
    x1, x2 = _np(X1).astype(np.float64), _np(X2).astype(np.float64)
    want = 0.95 * (x1.T @ x1 / rows) + 0.05 * (x2.T @ x2 / rows)
    assert _rel(_np(Fa), want) <= FACTOR_TOL
    assert torch.equal(Fa, Fa.T)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_band_split_all_bands_one_gpu(cuda, dt, world):
    """Every band of a world-rank split computed on one GPU (no NCCL): offset
    A operand (X + r0, transposed), band width r1 < d, the EMA epilogue on a
    band view; assembled and mirrored, against the fused kernel and the oracle."""
    from pytorch_opt_b200.dist import band_update_, kfac_band_bounds, mirror_lower_
    g = torch.Generator().manual_seed(31 + world)
    rows, d = 1024, 700  # d not a multiple of 16
    X1 = torch.randn(rows, d, generator=g).to(dt)
    X2 = torch.randn(rows, d, generator=g).to(dt)
    bounds = kfac_band_bounds(d, world)
    Fa = torch.empty(d, d, device=cuda)
    Fb = torch.empty(d, d, device=cuda)
    for X, first in ((X1, True), (X2, False)):
        Xc = X.to(cuda).contiguous()
        D = torch.zeros(d, d, device=cuda)
        for k in range(world):
            band_update_(D, Fa, Xc, 1.0 / rows, 0.95, first, bounds[k], bounds[k + 1])
        mirror_lower_(Fa, D)
        native.kron_syrk_ema_(Fb, Xc, 1.0 / rows, 0.95, first)
    assert _rel(_np(Fa), _np(Fb).astype(np.float64)) <= 1e-5
    x1, x2 = _np(X1).astype(np.float64), _np(X2).astype(np.float64)
    want = 0.95 * (x1.T @ x1 / rows) + 0.05 * (x2.T @ x2 / rows)
    assert _rel(_np(Fa), want) <= FACTOR_TOL
    assert torch.equal(Fa, Fa.T)


def test_kfac_golden_factors_and_inverse(cuda):
    """Golden KronTracker factors (ghat = n g) and the damped inverse by the Newton kernel."""
    z = np.load(os.path.join(GOLDEN_DIR, "kfac.npz"))
    for i in range(int(z["ncases"])):
        bias, ema = z[f"case{i}_meta"]
        if ema < 0:
            continue  # running-mean variant: same kernel with beta = count/(count+1)
        FA = torch.empty(6 + int(bias), 6 + int(bias), device=cuda)
        FG = torch.empty(5, 5, device=cuda)
        for step in range(3):
            a = torch.from_numpy(z[f"case{i}_a{step}"]).to(cuda)
            gr = torch.from_numpy(z[f"case{i}_g{step}"]).to(cuda)
            n = a.shape[0]
            if bias:
                a = torch.cat([a, torch.ones(n, 1, device=cuda)], dim=1)
            native.kron_syrk_ema_(FA, a, 1.0 / n, float(ema), step == 0)
            native.kron_syrk_ema_(FG, gr, float(n), float(ema), step == 0)  # ghat = n g: alpha = n^2 / n
        assert _rel(_np(FA), z[f"case{i}_A"]) <= FACTOR_TOL
        assert _rel(_np(FG), z[f"case{i}_G"]) <= FACTOR_TOL
        ga, _ = z[f"case{i}_gammas"]
        iA = native.damped_inverse(torch.from_numpy(z[f"case{i}_A"]).to(cuda), float(ga))
        assert _rel(_np(iA), z[f"case{i}_iA"]) <= 1e-4


def test_kfac_damped_inverse_large(cuda):
    g = torch.Generator(device=cuda).manual_seed(11)
    a = torch.randn(4096, 2048, device=cuda, generator=g)
    F = a.T @ a / 4096
    gamma = 1e-3
    X = native.damped_inverse(F, gamma)
    R = X.double() @ (F.double() + gamma * torch.eye(2048, device=cuda, dtype=torch.float64))
    R -= torch.eye(2048, device=cuda, dtype=torch.float64)
    assert float(R.norm() / math.sqrt(2048)) <= ROOT_TOL


def test_precond_golden_and_oracle(cuda):
    z = np.load(os.path.join(GOLDEN_DIR, "precond.npz"))
    for i in range(int(z["ncases"])):
        L, G, R = (torch.from_numpy(z[f"case{i}_{k}"]).to(cuda) for k in ("L", "G", "R"))
        assert _rel(_np(ops.precond_apply_two_sided(L, G, R)), z[f"case{i}_out"]) <= FACTOR_TOL
    g = torch.Generator().manual_seed(3)
    L, G, R = torch.randn(512, 512, generator=g), torch.randn(512, 300, generator=g), torch.randn(300, 300, generator=g)
    got = ops.precond_apply_two_sided(L.to(cuda), G.to(cuda), R.to(cuda))
    assert _rel(_np(got), O.precond_apply(_np(L).astype(np.float64), _np(G), _np(R))) <= FACTOR_TOL


@pytest.mark.parametrize("trans_l,trans_r", [(True, False), (False, True), (True, True)])
def test_rotate_two_sided_transposes_in_place(cuda, trans_l, trans_r):
    """op(QL) G op(QR) with transposed operands read in place (SOAP's rotations
    QL^T G QR and QL G QR^T), split-tf32: fp32-grade against fp64."""
    g = torch.Generator().manual_seed(17)
    m, n = 300, 520
    QL = torch.linalg.qr(torch.randn(m, m, generator=g, dtype=torch.float64))[0]
    QR = torch.linalg.qr(torch.randn(n, n, generator=g, dtype=torch.float64))[0]
    G = torch.randn(m, n, generator=g, dtype=torch.float64)
    got = native.rotate_two_sided(QL.float().to(cuda), G.float().to(cuda), QR.float().to(cuda), trans_l, trans_r)
    want = (QL.T if trans_l else QL) @ G @ (QR.T if trans_r else QR)
    assert _rel(_np(got), want.numpy()) <= 1e-5


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_precond_grafted_norm_from_epilogue(cuda, dt):
    """Grafting (shampoo.py:128-137): the epilogue's ||P||^2 matches the norm of
    the returned product and P * ratio matches the plain apply scaled on the host."""
    g = torch.Generator().manual_seed(4)
    L, G, R = torch.randn(640, 640, generator=g), torch.randn(640, 1100, generator=g), torch.randn(1100, 1100, generator=g)
    L, G, R = (t.to(cuda, dt) for t in (L, G, R))
    plain = native.precond_apply_two_sided(L, G, R)
    target = float(G.double().norm())
    P, ratio = native.precond_apply_grafted(L, G, R, target)
    # The epilogue sums the fp32 values before the output's rounding.
    want_ratio = target / (float(plain.double().norm()) + 1e-30)
    assert abs(float(ratio) - want_ratio) <= (1e-5 if dt == torch.float32 else 2e-3) * want_ratio
    np.testing.assert_allclose(_np(P), _np(plain) * float(ratio), rtol=1e-2 if dt == torch.bfloat16 else 1e-6,
                               atol=1e-30)


EKFAC_SCALE_TOL = 1e-4  # the running second moments: a factor-update-like statistic
# The output divides Vt by (s + damping): where Vt ~ sqrt(damping) the
# rounding of the split-bf16 products (~4e-6 relative in Vt) is amplified
# by up to ~1/(2 sqrt(damping)); measured 3e-5 .. 1.5e-4 against the
# reference's fp32 result and 6e-5 against fp64.
EKFAC_OUT_TOL = 5e-4


def test_ekfac_precondition_golden_and_oracle(cuda):
    """EKFAC (ekfac.py:44-58) on two consecutive gradients: the first call
    seeds the running scales, the second updates them in place."""
    z = np.load(os.path.join(GOLDEN_DIR, "ekfac.npz"))
    for i in range(int(z["ncases"])):
        decay, lam = (float(v) for v in z[f"case{i}_hp"])
        QG, QA = (torch.from_numpy(z[f"case{i}_{k}"]).to(cuda) for k in ("QG", "QA"))
        o1, s = native.ekfac_precondition(QG, QA, torch.from_numpy(z[f"case{i}_V1"]).to(cuda), None, decay, lam)
        assert _rel(_np(o1), z[f"case{i}_out1"]) <= EKFAC_OUT_TOL and _rel(_np(s), z[f"case{i}_s1"]) <= EKFAC_SCALE_TOL
        o2, s = native.ekfac_precondition(QG, QA, torch.from_numpy(z[f"case{i}_V2"]).to(cuda), s, decay, lam)
        assert _rel(_np(o2), z[f"case{i}_out2"]) <= EKFAC_OUT_TOL and _rel(_np(s), z[f"case{i}_s2"]) <= EKFAC_SCALE_TOL
    # A layer-sized case (ragged tiles, long K) against the oracle in fp64.
    g = torch.Generator().manual_seed(8)
    m, n = 700, 1300
    QG = torch.linalg.qr(torch.randn(m, m, generator=g, dtype=torch.float64))[0].float()
    QA = torch.linalg.qr(torch.randn(n, n, generator=g, dtype=torch.float64))[0].float()
    V1, V2 = torch.randn(m, n, generator=g), torch.randn(m, n, generator=g)
    o1, s = native.ekfac_precondition(QG.to(cuda), QA.to(cuda), V1.to(cuda), None, 0.95, 1e-3)
    o2, s = native.ekfac_precondition(QG.to(cuda), QA.to(cuda), V2.to(cuda), s, 0.95, 1e-3)
    w1, ws = O.ekfac_precondition(_np(QG).astype(np.float64), _np(QA), _np(V1), None, 0.95, 1e-3)
    w2, ws = O.ekfac_precondition(_np(QG).astype(np.float64), _np(QA), _np(V2), ws, 0.95, 1e-3)
    assert _rel(_np(o2), w2) <= EKFAC_OUT_TOL and _rel(_np(s), ws) <= EKFAC_SCALE_TOL


# ------------------------------------------------------------------------ Muon

def _bf16_ulps(got, want, ref_scale):
    """|got - want| in units of the bf16 spacing at max(|want|, |ref_scale|) (per element)."""
    w = np.maximum(np.abs(np.asarray(want, dtype=np.float64)), np.abs(np.asarray(ref_scale, dtype=np.float64)))
    spacing = np.exp2(np.floor(np.log2(np.maximum(w, 1e-30))) - 7)
    return np.abs(np.asarray(got, dtype=np.float64) - np.asarray(want, dtype=np.float64)) / spacing


def test_grouped_muon_golden(cuda):
    z = np.load(os.path.join(GOLDEN_DIR, "muon.npz"))
    lr, mom, nest, steps, wd = (float(v) for v in z["hparams"])
    groups = []
    for k in range(int(z["nparams"])):
        p = torch.from_numpy(z[f"p{k}_init"]).to(cuda, torch.bfloat16)[None].contiguous()
        groups.append(MuonGroup(p, torch.zeros_like(p)))
    opt = GroupedMuon(groups, lr=lr, momentum=mom, nesterov=bool(nest), ns_steps=int(steps), weight_decay=wd)
    for s in range(2):
        for k, grp in enumerate(groups):
            grp.grads.copy_(torch.from_numpy(z[f"p{k}_grad{s}"])[None])
        opt.step()
        assert abs(opt.update_rms() - float(z[f"update_rms{s}"])) <= NS_TOL * float(z[f"update_rms{s}"])
    for k, grp in enumerate(groups):
        np.testing.assert_array_equal(_np(grp.momentum[0]), z[f"p{k}_buf"])  # elementwise: bit-exact
        # The update is ~ a few bf16 ulps of p; NS differences within tolerance
        # can flip a rounding of p by one ulp per step.
        assert _bf16_ulps(_np(grp.params[0]), z[f"p{k}_final"], z[f"p{k}_init"]).max() <= 2.0


def test_grouped_muon_vs_oracle_gpt2_shapes(cuda):
    for shp in [(768, 2304), (768, 768), (3072, 768)]:
        g = torch.Generator().manual_seed(shp[1])
        p0 = (torch.randn(2, *shp, generator=g) * 0.02).bfloat16()
        gr = (torch.randn(2, *shp, generator=g) * 0.02).bfloat16()
        grp = MuonGroup(p0.clone().to(cuda), gr.clone().to(cuda), keep_update=True)
        GroupedMuon([grp], lr=0.02, weight_decay=0.01).step()
        for b in range(2):
            _, buf, Ow, _ = O.muon_matrix_step(_np(p0[b]), _np(gr[b]), np.zeros(shp, np.float32), lr=0.02,
                                               weight_decay=0.01)
            np.testing.assert_array_equal(_np(grp.momentum[b]), buf)  # elementwise: bit-exact
            O_gpu = _np(grp._u[b])
            assert _rel(O_gpu, Ow) <= NS_TOL  # the orthogonalised update itself
            # Given the kernel's O, the parameter update follows the reference's
            # in-place bf16 op sequence bit for bit (muon.py:87-91).
            p1 = O.bf16_round(_np(p0[b]) * np.float32(1.0 - 0.02 * 0.01))
            p2 = O.bf16_round(p1 + O.bf16_round(np.float32(-0.02 * O.muon_scale(shp))) * O_gpu)
            np.testing.assert_array_equal(_np(grp.params[b]), p2)


def test_sharded_step_from_host_equals_copy_then_step(cuda):
    """Host-to-device copies in batches (parts of groups) overlapped with the
    step give the same parameters, bit for bit, as one slot copy followed by
    the step."""
    from pytorch_opt_b200.dist import ShardLayout, ShardedMuon, host_copy_jobs
    shapes = [(768, 2304), (768, 768), (3072, 768), (768, 768), (256, 1024)] + [(2048, 2048)] * 9
    lay = ShardLayout(shapes, 1)
    jobs = host_copy_jobs([[(k, len(gr.indices), *gr.shape, 2) for k, gr in enumerate(lay.groups[0])]])[0]
    assert any(0 < s or e < len(lay.groups[0][k].indices) for k, s, e in jobs)  # some groups are split
    g = torch.Generator().manual_seed(9)
    p0 = (torch.randn(lay.numel, generator=g) * 0.02).bfloat16()
    host = (torch.randn(lay.slot, generator=g) * 0.02).bfloat16().pin_memory()
    out = []
    for use_host in (False, True):
        params = p0.clone().to(cuda)
        grads = torch.zeros(lay.numel, dtype=torch.bfloat16, device=cuda)
        sm = ShardedMuon(lay, params, grads, 0, lr=0.02, weight_decay=0.01)
        for _ in range(2):
            if use_host:
                sm.step_from_host(host)
            else:
                lay.load_slot(grads, 0, host)
                sm.step()
        torch.cuda.synchronize(cuda)
        out.append(params.cpu())
    assert torch.equal(out[0], out[1])



def _unfused_muon(p, g, buf, lr_eff, decay, steps=5):
    """momentum, Newton-Schulz and update as three C-ABI calls (the unfused sequence)."""
    lib = _lib.load()
    code = 1 if p.dtype == torch.bfloat16 else 0
    count, rows, cols = p.shape
    u = torch.empty_like(p)
    st = _lib.stream_ptr(p.device)
    _lib.check(lib.po_muon_momentum(g.data_ptr(), buf.data_ptr(), u.data_ptr(), code, u.numel(), 0.95, 1, st), "mom")
    nbytes = lib.po_ns_workspace_bytes(count, rows, cols)
    ws = _lib.workspace(nbytes, p.device)
    _lib.check(lib.po_newton_schulz(u.data_ptr(), code, count, rows, cols, cols, rows * cols, u.data_ptr(), cols,
                                    rows * cols, steps, 3.4445, -4.7750, 2.0315, 1e-7, -1, ws.data_ptr(), nbytes, st),
               "ns")
    sq = torch.zeros(1, dtype=torch.float64, device=p.device)
    _lib.check(lib.po_muon_apply(p.data_ptr(), u.data_ptr(), code, p.numel(), lr_eff, decay, sq.data_ptr(), st), "app")
    return u, sq


def _fused_muon(p, g, buf, lr_eff, decay, steps=5):
    lib = _lib.load()
    code = 1 if p.dtype == torch.bfloat16 else 0
    count, rows, cols = p.shape
    o = torch.empty_like(p)
    sq = torch.zeros(1, dtype=torch.float64, device=p.device)
    nbytes = lib.po_muon_step_workspace_bytes(count, rows, cols, code)
    ws = _lib.workspace(nbytes, p.device)
    _lib.check(lib.po_muon_step(g.data_ptr(), buf.data_ptr(), p.data_ptr(), code, count, rows, cols, 0.95, 1, steps,
                                3.4445, -4.7750, 2.0315, 1e-7, lr_eff, decay, sq.data_ptr(), o.data_ptr(),
                                ws.data_ptr(), nbytes, _lib.stream_ptr(p.device)), "po_muon_step")
    return o, sq


@pytest.mark.parametrize("shape,dt,steps", [
    ((3, 512, 1280), torch.bfloat16, 5),    # direct step 0 from u, wide
    ((2, 1280, 512), torch.bfloat16, 5),    # direct, tall (transposed operand and addend reads)
    ((2, 300, 522), torch.bfloat16, 5),     # row pitch not 16-byte aligned: packed step 0
    ((2, 96, 200), torch.bfloat16, 5),      # small m: split-bf16 schedule
    ((2, 384, 640), torch.float32, 5),      # fp32 parameters
    ((2, 512, 768), torch.bfloat16, 1),     # one step: the first update is also the last
    ((1, 64, 96), torch.bfloat16, 0),       # no step: O is the normalised u
])
def test_fused_muon_step_vs_unfused(cuda, shape, dt, steps):
    """po_muon_step against momentum + Newton-Schulz + update as separate calls:
    momentum bit-exact; O within the Newton-Schulz tolerance (step 0 reads u
    unrounded-by-scaling, the unfused path packs a rounded copy of u/||u||);
    the parameter update bit-exact given the fused call's own O (the
    reference's in-place op sequence, muon.py:87-91); sum(O^2) consistent."""
    g = torch.Generator().manual_seed(sum(shape) + steps)
    p0 = (torch.randn(*shape, generator=g) * 0.02).to(dt)
    gr = (torch.randn(*shape, generator=g) * 0.02).to(dt)
    b0 = (torch.randn(*shape, generator=g) * 0.02).to(dt)
    lr_eff, decay = 0.02 * max(1.0, shape[1] / shape[2]) ** 0.5, 1.0 - 0.02 * 0.01
    pu, bu = p0.to(cuda), b0.to(cuda)
    pf, bf = p0.to(cuda), b0.to(cuda)
    Ou, squ = _unfused_muon(pu, gr.to(cuda), bu, lr_eff, decay, steps)
    Of, sqf = _fused_muon(pf, gr.to(cuda), bf, lr_eff, decay, steps)
    assert torch.equal(bu, bf)
    assert _rel(_np(Of), _np(Ou)) <= NS_TOL
    p1 = _np(p0) * np.float32(decay)
    if dt == torch.bfloat16:
        p1 = O.bf16_round(p1)
        alpha = O.bf16_round(np.float32(-lr_eff))
        want_p = O.bf16_round(p1 + alpha * _np(Of))
    else:
        want_p = p1 + np.float32(-lr_eff) * _np(Of)
    if dt == torch.bfloat16:  # alpha and O are bf16: alpha * O is exact in fp32, one rounding as in the kernel
        np.testing.assert_array_equal(_np(pf), want_p)
    else:
        np.testing.assert_allclose(_np(pf), want_p, rtol=1e-6, atol=1e-9)
    sq_want = float((Of.double() ** 2).sum())
    assert abs(float(sqf) - sq_want) <= 1e-5 * sq_want
