"""Host-side checks that need no GPU: the C ABI's exports and argument
validation, the ops-API mirror's error behaviour, and the sharding plan."""

import ctypes
import os
import re

import pytest
import torch

from pytorch_opt_b200 import _lib, native, ops
from pytorch_opt_b200.dist import ShardLayout, lpt_assign, ns_flops
from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "pytorch_opt_b200.h")


def _header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(po_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = _header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    # the ctypes binding declares exactly the header's functions
    assert set(_lib.SIGNATURES) == set(names)


def test_load_and_version():
    lib = _lib.load()
    assert b"sm_100a" in lib.po_version()


def test_abi_rejects_bad_arguments_without_touching_the_device():
    lib = _lib.load()
    # bad dtype
    assert lib.po_newton_schulz(None, 7, 1, 4, 4, 4, 16, None, 4, 16, 5, 3.4, -4.7, 2.0, 1e-7, -1, None, 0,
                                None) == 1
    assert "dtype" in _lib.last_error()
    # negative sizes
    assert lib.po_newton_schulz(None, 0, 1, -4, 4, 4, 16, None, 4, 16, 5, 3.4, -4.7, 2.0, 1e-7, -1, None, 0,
                                None) == 1
    # empty problems are no-ops
    assert lib.po_newton_schulz(None, 0, 0, 4, 4, 4, 16, None, 4, 16, 5, 3.4, -4.7, 2.0, 1e-7, -1, None, 0,
                                None) == 0
    # p must be a positive integer (reference: ValueError / TORCH_CHECK)
    assert lib.po_inverse_root(None, 0, 1, 4, 4, 16, None, 4, 16, 0, 0.0, 100, 1e-10, None, None, 0, None) == 1
    assert "positive integer" in _lib.last_error()
    # workspace too small is reported, not written past
    assert lib.po_newton_schulz(ctypes.c_void_p(16), 0, 1, 4, 4, 4, 16, ctypes.c_void_p(16), 4, 16, 5, 3.4, -4.7,
                                2.0, 1e-7, -1, ctypes.c_void_p(256), 8, None) == 3
    assert "workspace" in _lib.last_error()
    assert lib.po_matmul(None, 1, 1, 0, None, 1, 1, 0, None, 1, 1, 0, 0, 1, 1, 1, 0, 1.0, 0.0, None, 0, None) == 5


def test_workspace_sizes_are_consistent():
    lib = _lib.load()
    a = lib.po_ns_workspace_bytes(1, 768, 3072)
    assert a == lib.po_ns_workspace_bytes(1, 3072, 768)  # transposed problem, same work
    assert lib.po_ns_workspace_bytes(2, 768, 3072) > a
    assert lib.po_ns_workspace_bytes(0, 8, 8) == 0
    r4 = lib.po_root_workspace_bytes(8, 1024, 4)
    r1 = lib.po_root_workspace_bytes(8, 1024, 1)
    assert r4 > r1 > 0
    assert lib.po_syrk_workspace_bytes(8192, 4096, 1) < lib.po_syrk_workspace_bytes(8192, 4096, 0)


def test_ops_mirror_argument_errors():
    A = torch.eye(3)
    with pytest.raises(ValueError, match="positive integer"):
        ops.inverse_matrix_root(A, 0)
    with pytest.raises(ValueError, match="method"):
        ops.inverse_matrix_root(A, 2, method="qr")
    with pytest.raises(ValueError, match="ndim"):
        ops.newton_schulz_orthogonalize(torch.ones(3))
    with pytest.raises(ValueError, match="2D"):
        ops.kron_factor_update_(torch.zeros(2, 2), torch.zeros(2, 2), torch.zeros(2, 2, 2))


def test_ops_mirror_backend_switch():
    assert ops.get_backend() == "auto"
    with pytest.raises(ValueError, match="backend"):
        ops.set_backend("bogus")
    with pytest.raises(RuntimeError, match="native backend only"):
        ops.set_backend("reference")
    assert ops.load_native() is True and ops.native_available()
    ops.set_backend("native")
    assert ops.get_backend() == "native"
    ops.set_backend("auto")


def test_no_cpu_fallback():
    """CPU tensors are refused loudly: the native path never computes on the host."""
    ops.load_native()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.newton_schulz_orthogonalize(torch.randn(8, 5))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        native.inverse_matrix_root(torch.eye(4), 4, 0.0, "newton", True, 100, 1e-10)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        native.kron_factor_update_(torch.zeros(2, 2), torch.zeros(3, 3), torch.zeros(2, 3), 1.0)
    with pytest.raises(RuntimeError, match="positive integer"):
        native.inverse_matrix_root(torch.eye(4), 0, 0.0, "newton", True, 100, 1e-10)
    with pytest.raises(RuntimeError, match="method"):
        native.inverse_matrix_root(torch.eye(4), 2, 0.0, "qr", True, 100, 1e-10)


LLAMA = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)] * 32


def test_lpt_assignment_balances_llama_matrices():
    costs = [ns_flops(r, c) for r, c in LLAMA]
    for world in (1, 2, 4, 8):
        plan = lpt_assign(costs, world)
        assert sorted(i for part in plan for i in part) == list(range(len(LLAMA)))
        loads = [sum(costs[i] for i in part) for part in plan]
        assert max(loads) <= sum(costs) / world + max(costs)  # LPT bound
        assert max(loads) / (sum(costs) / world) < 1.06
        assert plan == lpt_assign(costs, world)  # deterministic on every rank


def test_shard_layout_is_disjoint_and_grouped():
    shapes = [(64, 96), (96, 64), (64, 96), (32, 32), (64, 96), (16, 48)]
    for world, chunks in ((1, None), (2, None), (3, 2), (2, 5)):
        lay = ShardLayout(shapes, world, chunks=chunks)
        flat = torch.zeros(lay.numel)
        seen = torch.zeros(lay.numel, dtype=torch.int32)
        for i, (r, c) in enumerate(shapes):
            v = lay.matrix(flat, i)
            assert tuple(v.shape) == (r, c)
            rank, off = lay.offset_of[i]
            parts = [(lay.chunk_base[k] + rank * lay.chunk_len[k], lay.chunk_len[k]) for k in range(lay.chunks)]
            assert any(s <= off and off + r * c <= s + n for s, n in parts)  # inside one of its rank's chunk parts
            seen[off:off + r * c] += 1
        assert int(seen.max()) == 1
        for rank in range(world):
            for g, v in zip(lay.groups[rank], lay.group_views(flat, rank)):
                assert tuple(v.shape) == (len(g.indices), *g.shape)
                for k, i in enumerate(g.indices):  # group view k is matrix i
                    assert v[k].data_ptr() == lay.matrix(flat, i).data_ptr()


def test_step_from_host_matches_copy_then_step_on_cpu():
    """The host-gradient step (per-group copies) equals copying the slot and stepping."""
    from pytorch_opt_b200.dist import ShardedMuon
    shapes = [(64, 96), (96, 64), (64, 96), (32, 32), (16, 48)]
    lay = ShardLayout(shapes, 1)
    g = torch.Generator().manual_seed(3)
    host = torch.randn(lay.slot, generator=g)

    def fake_update(p, grad):
        p.add_(grad * 0.5 + 1.0)

    out = []
    for use_host in (False, True):
        params = torch.zeros(lay.numel)
        grads = torch.zeros(lay.numel)
        sm = ShardedMuon(lay, params, grads, 0, compute=fake_update)
        if use_host:
            sm.step_from_host(host)
        else:
            lay.load_slot(grads, 0, host)
            sm.step()
        out.append(params.clone())
    assert torch.equal(out[0], out[1])
    with pytest.raises(ValueError):
        ShardedMuon(lay, torch.zeros(lay.numel), torch.zeros(lay.numel), 0, compute=fake_update).step_from_host(
            host[:-1])


def test_host_copy_jobs_expose_only_the_first_matrix_copy():
    """Host-gradient batches (Johnson's order, sized to the copy stream's
    lead) cover every matrix once, and in a copy-then-compute flow shop with
    the Llama-3-8B groups only the first (one-matrix) copy is left without
    compute to hide it."""
    from pytorch_opt_b200.dist import H2D_BYTES_PER_FLOP, host_copy_jobs, ns_executed_flops as ns_flops
    groups = [(0, 64, 4096, 4096, 2), (1, 64, 1024, 4096, 2), (2, 64, 14336, 4096, 2), (3, 32, 4096, 14336, 2)]
    for split in ([groups], [groups[:2], groups[2:]]):
        jobs = [j for c in host_copy_jobs(split) for j in c]
        seen = {k: [] for k, *_ in groups}
        for k, s, e in jobs:
            assert 0 < e - s <= 32
            seen[k].extend(range(s, e))
        assert all(sorted(v) == list(range(groups[k][1])) for k, v in seen.items())
        assert jobs[0][2] - jobs[0][1] == 1
        shape = {k: (r, c, es) for k, _, r, c, es in groups}
        copy_end = compute_end = busy = 0.0
        for i, (k, s, e) in enumerate(jobs):
            r, c, es = shape[k]
            a = (e - s) * r * c * es
            b = (e - s) * ns_flops(r, c) * H2D_BYTES_PER_FLOP
            copy_end += a
            compute_end = max(compute_end, copy_end) + b
            busy += b
            if i == 0:
                first_copy = a
        assert compute_end - busy <= first_copy * (1 + 1e-9)
    jobs = host_copy_jobs([groups])[0]
    assert len(jobs) <= 16
    kinds = [shape[k][0] == 1024 for k, _, _ in jobs]  # copy-bound batches (k/v) come last
    assert kinds == sorted(kinds)


def test_kfac_band_bounds_balance_the_triangle():
    from pytorch_opt_b200.dist import kfac_band_bounds
    for d in (4096, 1000, 300):
        for world in (1, 2, 3, 4, 8):
            b = kfac_band_bounds(d, world)
            assert b[0] == 0 and b[-1] == d and len(b) == world + 1
            assert all(x <= y for x, y in zip(b, b[1:]))
            assert all(x % 16 == 0 or x == d for x in b[1:-1])
            work = [(y - x) * y for x, y in zip(b, b[1:])]  # band rectangle areas
            if d == 4096:
                assert max(work) <= 1.05 * sum(work) / world
                assert sum(work) <= d * d  # never more than the full square



def test_exchange_chunks_end_with_the_cheapest_exchange():
    """Exchange chunks have decreasing FLOP shares, and within every rank the
    matrices are ordered by decreasing exchanged bytes per FLOP, so the last
    chunk (whose all-gather cannot overlap compute) is small and holds the
    matrices that are cheapest to exchange (Llama: q/o at N = 8)."""
    from pytorch_opt_b200.dist import ShardLayout, bytes_per_flop, chunk_shares, ns_flops
    shares = chunk_shares(4)
    assert abs(sum(shares) - 1.0) < 1e-12 and all(a > b for a, b in zip(shares, shares[1:]))
    layer = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
    for world in (2, 4, 8):
        lay = ShardLayout(layer * 32, world)
        seen = set()
        for r in range(world):
            per_chunk_flops = [0.0] * lay.chunks
            worst_bpf = [0.0] * lay.chunks
            for g in lay.groups[r]:
                per_chunk_flops[g.chunk] += ns_flops(*g.shape) * len(g.indices)
                worst_bpf[g.chunk] = max(worst_bpf[g.chunk], bytes_per_flop(*g.shape))
                seen.update(g.indices)
            assert per_chunk_flops[-1] <= 0.15 * sum(per_chunk_flops)
            assert worst_bpf[-1] <= min(w for w in worst_bpf if w > 0)  # the last chunk is cheapest to exchange
        assert seen == set(range(len(layer) * 32))
