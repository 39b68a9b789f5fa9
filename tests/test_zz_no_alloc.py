"""The allocation-free Newton–Schulz entry point (po_newton_schulz_static).

Some callers cannot allocate device memory: code running inside a framework
that owns every byte of device memory through its own pool, or plug-in code
that is handed device pointers but no allocator. ``po_newton_schulz_static``
serves them from a fixed scratch array inside the library. These tests call
it through the C ABI twice in a row (the scratch keeps the previous call's
contents) and compare each result with the workspace-taking
``po_newton_schulz`` on the same input: both run the same kernels, so they
must agree to 1e-6 (the per-matrix norm is summed with atomics, whose order
may move its last bits). Each result is also checked against the numpy
oracle within the Newton–Schulz tolerance of the parity tests (1e-2
relative Frobenius). A problem larger than the scratch must be refused with
a clear error. This file is collected last.
"""

import numpy as np
import pytest
import torch

from oracle import ops_np as O
from pytorch_opt_b200 import _lib

pytestmark = pytest.mark.gpu

NS_TOL = 1e-2
SAME_KERNELS_TOL = 1e-6
COEFFS = (3.4445, -4.7750, 2.0315)
CODE = {torch.float32: 0, torch.bfloat16: 1}


def _with_workspace(G: torch.Tensor) -> torch.Tensor:
    lib = _lib.load()
    b, r, c = G.shape
    out = torch.empty_like(G)
    nbytes = lib.po_ns_workspace_bytes(b, r, c)
    ws = _lib.workspace(nbytes, G.device)
    _lib.check(lib.po_newton_schulz(G.data_ptr(), CODE[G.dtype], b, r, c, c, r * c, out.data_ptr(), c, r * c, 5,
                                    *COEFFS, 1e-7, -1, ws.data_ptr(), nbytes, _lib.stream_ptr(G.device)),
               "po_newton_schulz")
    return out


def _without_allocation(G: torch.Tensor) -> tuple[int, torch.Tensor]:
    lib = _lib.load()
    b, r, c = G.shape
    out = torch.empty_like(G)
    rc = lib.po_newton_schulz_static(G.data_ptr(), CODE[G.dtype], b, r, c, c, r * c, out.data_ptr(), c, r * c, 5,
                                     *COEFFS, 1e-7, -1, _lib.stream_ptr(G.device))
    return rc, out


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.double(), b.double()
    return float((a64 - b64).norm() / b64.norm())


def test_static_scratch_matches_workspace_entry_twice(cuda):
    g = torch.Generator(device=cuda).manual_seed(123)
    first = torch.randn(1, 1024, 1024, device=cuda, generator=g)                    # fills most of the scratch
    second = (torch.randn(3, 200, 96, device=cuda, generator=g) * 0.02).bfloat16()  # tall, batched, other schedule
    for G in (first, second):
        rc, got = _without_allocation(G)
        assert rc == 0, _lib.last_error()
        want = _with_workspace(G)
        torch.cuda.synchronize(cuda)
        assert _rel(got, want) <= SAME_KERNELS_TOL, _rel(got, want)
        assert torch.isfinite(got.float()).all()
        x = G.float().cpu().numpy()
        oracle = O.newton_schulz(x, 5, out_bf16=(G.dtype == torch.bfloat16))
        got64 = got.double().cpu().numpy()
        assert np.linalg.norm(got64 - oracle) / np.linalg.norm(oracle) <= NS_TOL
    assert _lib.device_error(reset=True) == 0


def test_static_scratch_rejects_oversized_problem(cuda):
    lib = _lib.load()
    need = lib.po_ns_workspace_bytes(1, 4096, 4096)
    assert need > 32 << 20
    G = torch.zeros(1, 1, 1, device=cuda)  # never read: the size check comes first
    rc = lib.po_newton_schulz_static(G.data_ptr(), 0, 1, 4096, 4096, 4096, 4096 * 4096, G.data_ptr(), 4096,
                                     4096 * 4096, 5, *COEFFS, 1e-7, -1, None)
    assert rc == 1
    msg = _lib.last_error()
    assert "scratch" in msg and str(need) in msg
