"""GPU tests of the tcgen05 product kernel underneath every op, through the
exported ``po_matmul`` C-ABI entry point: the one-SM kernel (128-row tiles)
and the two-SM kernel (256 x 256 tiles on a cluster of two CTAs), forced in
turn with ``PO_GEMM_PAIR``, on all four operand layouts, both operand kinds,
ragged shapes (partial tiles in M, N and K) and batches.

Reference: float64 matmul of the operands as the tensor cores see them
(bf16 exactly; fp32 inputs rounded to tf32 by truncation for precision 0,
exact for the split precisions 1 and 2). Tolerances, relative Frobenius:
bf16 and split-bf16 2e-5 (fp32 accumulation over K <= 1100), split-tf32
2e-6, tf32 2e-3 (10-bit mantissa operands).
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import ops_np as O
from pytorch_opt_b200 import _lib, native

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_error_stays_clear(cuda):
    yield
    assert _lib.device_error(reset=True) == 0


def _tf32_trunc(x: torch.Tensor) -> torch.Tensor:
    return (x.contiguous().view(torch.int32) & ~0x1FFF).view(torch.float32)


def _matmul(A, B, C, ta, tb, precision, alpha, beta):
    """C = alpha op(A) op(B) + beta C via po_matmul (A, B, C: [batch, r, c])."""
    lib = _lib.load()
    batch = A.shape[0]
    M, K = (A.shape[2], A.shape[1]) if ta else (A.shape[1], A.shape[2])
    N = B.shape[1] if tb else B.shape[2]
    dtype = 1 if A.dtype == torch.bfloat16 else 0
    nbytes = lib.po_matmul_workspace_bytes(batch, M, N, K, dtype, precision)
    ws = _lib.workspace(nbytes, A.device)
    rc = lib.po_matmul(A.data_ptr(), A.stride(1), A.stride(0), ta, B.data_ptr(), B.stride(1), B.stride(0), tb,
                       ctypes.c_void_p(C.data_ptr()), C.stride(1), C.stride(0), dtype, precision, batch, M, N, K,
                       alpha, beta, ws.data_ptr(), nbytes, _lib.stream_ptr(A.device))
    _lib.check(rc, "po_matmul")


def _reference(A, B, C0, ta, tb, precision, alpha, beta):
    a = A.double() if A.dtype == torch.bfloat16 or precision >= 1 else _tf32_trunc(A).double()
    b = B.double() if B.dtype == torch.bfloat16 or precision >= 1 else _tf32_trunc(B).double()
    if ta:
        a = a.transpose(1, 2)
    if tb:
        b = b.transpose(1, 2)
    return alpha * (a @ b) + beta * C0.double()


def _rel(x, y):
    return float((x.double() - y).norm() / y.norm().clamp_min(1e-300))


LAYOUTS = [(0, 0), (0, 1), (1, 0), (1, 1)]
# (bf16, 1): bf16 products whose K is summed in chunks outside the accumulator;
# (fp32, 1): split-bf16 pairs; (fp32, 2): split-tf32 pairs (fp32-grade).
KINDS = [(torch.bfloat16, 0, 2e-5), (torch.bfloat16, 1, 2e-5), (torch.float32, 0, 2e-3), (torch.float32, 1, 2e-5),
         (torch.float32, 2, 2e-6)]


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("ta,tb", LAYOUTS)
@pytest.mark.parametrize("dt,precision,tol", KINDS)
def test_matmul_layouts_ragged(cuda, monkeypatch, pair, ta, tb, dt, precision, tol):
    monkeypatch.setenv("PO_GEMM_PAIR", pair)
    g = torch.Generator(device="cpu").manual_seed(1000 + 4 * ta + 2 * tb + precision)
    batch, M, N, K = 2, 300, 520, 1096
    a_shape = (batch, K, M) if ta else (batch, M, K)
    b_shape = (batch, N, K) if tb else (batch, K, N)
    A = torch.randn(a_shape, generator=g).to(cuda, dt)
    B = torch.randn(b_shape, generator=g).to(cuda, dt)
    C0 = torch.randn((batch, M, N), generator=g).to(cuda)
    C = C0.clone()
    _matmul(A, B, C, ta, tb, precision, 0.75, 0.5)
    want = _reference(A, B, C0, ta, tb, precision, 0.75, 0.5)
    assert _rel(C, want) <= tol


@pytest.mark.parametrize("dt,precision", [(torch.bfloat16, 0), (torch.float32, 0)])
def test_pair_and_single_sm_tiles_agree(cuda, monkeypatch, dt, precision):
    """Both tile shapes run the same k order per output element: results agree
    to fp32 rounding (in practice bit for bit)."""
    g = torch.Generator(device="cpu").manual_seed(7)
    A = torch.randn((1, 1024, 768), generator=g).to(cuda, dt)
    B = torch.randn((1, 768, 1280), generator=g).to(cuda, dt)
    out = {}
    for pair in ("0", "1"):
        monkeypatch.setenv("PO_GEMM_PAIR", pair)
        C = torch.zeros((1, 1024, 1280), device=cuda)
        _matmul(A, B, C, 0, 0, precision, 1.0, 0.0)
        out[pair] = C
    assert _rel(out["1"], out["0"].double()) <= 1e-6


def test_pair_kernel_is_launched(cuda, monkeypatch):
    """With the pair path forced, the two-SM kernel is the one that runs."""
    monkeypatch.setenv("PO_GEMM_PAIR", "1")
    A = torch.randn((1, 512, 512), device=cuda).bfloat16()
    B = torch.randn((1, 512, 512), device=cuda).bfloat16()
    C = torch.zeros((1, 512, 512), device=cuda)
    _matmul(A, B, C, 0, 0, 0, 1.0, 0.0)  # first call configures the kernel
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        _matmul(A, B, C, 0, 0, 0, 1.0, 0.0)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("tc_gemm_pair_kernel" in n for n in names), names


@pytest.mark.parametrize("shape", [(512, 512), (768, 2048), (1024, 1024)])
def test_ns_on_pair_tiles_vs_oracle(cuda, monkeypatch, shape):
    """Newton-Schulz (triangular Gram / square products with mirrored stores,
    fused update epilogue) on two-SM tiles, against the numpy oracle."""
    monkeypatch.setenv("PO_GEMM_PAIR", "1")
    rng = np.random.default_rng(11)
    G = rng.standard_normal(shape).astype(np.float32)
    got = native.newton_schulz_orthogonalize(torch.from_numpy(G).to(cuda), 5, 3.4445, -4.7750, 2.0315, 1e-7)
    want = O.newton_schulz(G, 5, (3.4445, -4.7750, 2.0315), 1e-7)
    rel = float(np.linalg.norm(got.double().cpu().numpy() - want) / np.linalg.norm(want))
    assert rel <= 1e-2


def test_root_on_pair_tiles(cuda, monkeypatch):
    """Coupled-Newton inverse 4th root (diagonal-split epilogue) on two-SM tiles."""
    monkeypatch.setenv("PO_GEMM_PAIR", "1")
    rng = np.random.default_rng(5)
    X = rng.standard_normal((2048, 640))
    A = (X.T @ X / 2048).astype(np.float32)
    out = native.inverse_matrix_root(torch.from_numpy(A).to(cuda), 4, 1e-6, "newton", False, 100, 1e-6)
    res = O.root_residual(out.double().cpu().numpy(), A.astype(np.float64), 4, 1e-6)
    assert res <= 1e-4


def test_root_batched_mixed_conditioning_on_pair_tiles(cuda, monkeypatch):
    """Items that converge at different iterations are skipped by later
    launches (per-item active flags and pass counts) while the other items'
    tiles keep flowing through the two-SM kernel's dynamic tile queue."""
    monkeypatch.setenv("PO_GEMM_PAIR", "1")
    rng = np.random.default_rng(17)
    d = 600  # ragged: three 256-row tiles, the last one partial
    mats = []
    for k, scale in enumerate((1.0, 40.0, 0.0)):
        if scale == 0.0:
            mats.append(np.eye(d) * 3.0)  # converges at once
            continue
        X = rng.standard_normal((2 * d, d))
        mats.append(X.T @ X / (2 * d) * scale + 1e-3 * np.eye(d))
    A = torch.from_numpy(np.stack(mats).astype(np.float32)).to(cuda)
    out = native.inverse_matrix_root(A, 4, 1e-6, "newton", False, 100, 1e-6)
    for i, M in enumerate(mats):
        assert O.root_residual(out[i].double().cpu().numpy(), M.astype(np.float32).astype(np.float64), 4, 1e-6) <= 1e-4


@pytest.mark.parametrize("shape", [(3, 640, 1664), (2, 1400, 520)])
def test_ns_batched_ragged_on_pair_tiles(cuda, monkeypatch, shape):
    """Batched, ragged and tall (transposed) Newton-Schulz on two-SM tiles."""
    monkeypatch.setenv("PO_GEMM_PAIR", "1")
    rng = np.random.default_rng(23)
    G = rng.standard_normal(shape).astype(np.float32)
    got = native.newton_schulz_orthogonalize(torch.from_numpy(G).to(cuda), 5, 3.4445, -4.7750, 2.0315, 1e-7)
    for b in range(shape[0]):
        want = O.newton_schulz(G[b], 5, (3.4445, -4.7750, 2.0315), 1e-7)
        rel = float(np.linalg.norm(got[b].double().cpu().numpy() - want) / np.linalg.norm(want))
        assert rel <= 1e-2

