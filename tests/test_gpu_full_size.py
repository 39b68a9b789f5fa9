"""GPU parity at the benchmark configurations' full problem sizes.

The kernels are compared with the reference algorithm evaluated by torch on
the same GPU (``oracle.ops_torch``: fp32 products without TF32 for
Newton–Schulz, as the reference computes; fp64 for roots and KFAC factors),
and that checker is itself pinned to the reference's own full-size outputs:
``tests/golden/full_size.npz`` holds 32 x 32 two-sided sketches L^T X R of
what the reference computed on the identical seeded inputs
(``tests/golden/make_full_size.py``), and its iteration counts and KFAC
condition numbers.

Tolerances: Newton–Schulz relative Frobenius error <= 1e-2; roots residual
||X^4 (A + eps I) - I||_F / sqrt(d) <= 1e-4 and the reference's iteration
count; KFAC factors relative error <= 1e-4; damped inverse residual
||X (F + gamma I) - I||_F / sqrt(d) <= 1e-4. Each test prints what it
measured.
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import ops_torch as T
from pytorch_opt_b200 import _lib, native, ops
from tests.conftest import GOLDEN_DIR
from tests.golden.make_full_size import NS_SHAPES, ROOT_DIMS, kfac_batch, ns_input, shampoo_factor

pytestmark = pytest.mark.gpu

NS_TOL = 1e-2
ROOT_TOL = 1e-4
FACTOR_TOL = 1e-4
FULL = np.load(os.path.join(GOLDEN_DIR, "full_size.npz"))


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.double(), b.double()
    return float((a64 - b64).norm() / b64.norm())


def _sk_rel(sk: torch.Tensor, ref: np.ndarray) -> float:
    r = torch.from_numpy(ref).to(sk.device)
    return float((sk - r).norm() / r.norm())


@pytest.fixture(autouse=True)
def _device_error_stays_clear(cuda):
    yield
    assert _lib.device_error(reset=True) == 0


@pytest.mark.parametrize("i", range(len(NS_SHAPES)), ids=[f"{r}x{c}" for r, c in NS_SHAPES])
def test_ns_full_size_llama_shapes(cuda, i):
    """Config-5 shapes (bf16 0.02 N(0,1), seed 1000 + i) against the reference's fp32 NS5."""
    rows, cols, _, ls, rs = (int(v) for v in FULL[f"ns{i}_meta"])
    G = ns_input(i).to(cuda)
    got = ops.newton_schulz_orthogonalize(G)
    assert got.dtype == torch.bfloat16 and got.shape == (rows, cols)
    with T.exact_fp32_matmul():
        want32 = T.newton_schulz(G.float())  # the reference's fp32 work, before its cast back to bf16
        sk32 = T.two_sided_sketch(want32, ls, rs)
        # The GPU checker reproduces the reference's own code run in fp64.
        err_checker = _sk_rel(sk32, FULL[f"ns{i}_sketch_f64"])
        want = want32.bfloat16()  # what the reference returns for bf16 input (reference.py:97)
        err_full = _rel(got, want)
        sk = T.two_sided_sketch(got, ls, rs)
        err_sketch = _sk_rel(sk, FULL[f"ns{i}_sketch"])  # the reference's own bf16 result on the CPU
        err_f64 = _sk_rel(sk, FULL[f"ns{i}_sketch_f64"])
    # The reference's CPU fp32 run sums its Frobenius norm in fp32 (0.5 % low
    # at 14336 x 4096), so its output differs from its own fp64 run by up to ~5e-3.
    ref32_vs_64 = float(np.linalg.norm(FULL[f"ns{i}_sketch_f32"] - FULL[f"ns{i}_sketch_f64"])
                        / np.linalg.norm(FULL[f"ns{i}_sketch_f64"]))
    print(f"NS {rows}x{cols}: rel Frobenius {err_full:.3e} vs fp32 torch on the GPU; vs the reference's bf16 "
          f"output {err_sketch:.3e}, vs the reference in fp64 {err_f64:.3e} (sketches); checker vs reference fp64 "
          f"{err_checker:.1e}; reference fp32 vs its fp64 {ref32_vs_64:.1e}")
    assert err_checker <= 5e-4, err_checker
    assert err_full <= NS_TOL, err_full
    assert err_sketch <= NS_TOL, err_sketch
    assert err_f64 <= NS_TOL, err_f64


@pytest.mark.parametrize("d", ROOT_DIMS)
def test_root_full_size_iterations_and_residual(cuda, d):
    """Config-3 factors: same iteration count as the reference's fp64 loop, residual, and closeness."""
    L = shampoo_factor(d).to(cuda)
    lib = _lib.load()
    out = torch.empty_like(L)
    its = torch.zeros(1, dtype=torch.int32, device=cuda)
    nbytes = lib.po_root_workspace_bytes(1, d, 4)
    ws = _lib.workspace(nbytes, cuda)
    _lib.check(lib.po_inverse_root(L.data_ptr(), 0, 1, d, d, d * d, out.data_ptr(), d, d * d, 4, 1e-8, 100, 1e-10,
                                   its.data_ptr(), ws.data_ptr(), nbytes, _lib.stream_ptr(cuda)), "root")
    want, its_checker = T.inverse_root_newton(L, 4, 1e-8)
    its_ref = int(FULL[f"root{d}_iters"])
    err_checker = _sk_rel(T.two_sided_sketch(want.float(), 7100 + d, 8100 + d), FULL[f"root{d}_sketch"])
    res = T.root_residual(out, L, 4, 1e-8)
    err = _rel(out, want)
    print(f"root d={d}: iterations {int(its.item())} (reference {its_ref}), residual {res:.3e}, rel {err:.3e} "
          f"(checker vs reference {err_checker:.1e})")
    assert its_checker == its_ref and err_checker <= 1e-6
    assert int(its.item()) == its_ref
    assert res <= ROOT_TOL
    assert err <= 1e-4


def test_kfac_full_size_factors_and_inverses(cuda):
    """Config 4: SYRK+EMA of A and G from two 8192 x 4096 bf16 batches, pi-damped Newton inverses."""
    n = 8192
    FA = torch.empty(4096, 4096, device=cuda)
    FG = torch.empty(4096, 4096, device=cuda)
    A_ref = G_ref = None
    for step, (sa, sg) in enumerate([(1, 2), (3, 4)]):
        a, g = kfac_batch(sa).to(cuda), kfac_batch(sg).to(cuda)
        native.kron_syrk_ema_(FA, a, 1.0 / n, 0.95, step == 0)
        native.kron_syrk_ema_(FG, g, float(n), 0.95, step == 0)
        A_ref = T.kfac_update(A_ref, T.kron_batch_factor(a, 1.0 / n), 0.95)
        G_ref = T.kfac_update(G_ref, T.kron_batch_factor(g, float(n)), 0.95)
        ea, eg = _rel(FA, A_ref), _rel(FG, G_ref)
        ca = _sk_rel(T.two_sided_sketch(A_ref, 7200 + step, 8200 + step), FULL[f"kfac_A{step}_sketch"])
        cg = _sk_rel(T.two_sided_sketch(G_ref, 7300 + step, 8300 + step), FULL[f"kfac_G{step}_sketch"])
        print(f"KFAC step {step}: A rel {ea:.3e}, G rel {eg:.3e} (checker vs reference {ca:.1e}, {cg:.1e})")
        assert ca <= 1e-5 and cg <= 1e-5
        assert ea <= FACTOR_TOL and eg <= FACTOR_TOL
        assert torch.equal(FA, FA.T) and torch.equal(FG, FG.T)
    ga, gg = (float(v) for v in FULL["kfac_gammas"])
    eye = torch.eye(4096, device=cuda, dtype=torch.float64)
    for name, F, gamma, key in (("A", FA, ga, "iA"), ("G", FG, gg, "iG")):
        X = native.damped_inverse(F, gamma)
        res = float((X.double() @ (F.double() + gamma * eye) - eye).norm() / math.sqrt(4096))
        sk = _sk_rel(T.two_sided_sketch(X, 7400 if key == "iA" else 7500, 8400 if key == "iA" else 8500),
                     FULL[f"kfac_{key}_sketch"])
        print(f"KFAC damped inverse {name}: residual {res:.3e}, sketch vs reference eigh inverse {sk:.3e}")
        assert res <= ROOT_TOL
        assert sk <= 1e-4
