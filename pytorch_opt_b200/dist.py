"""Per-matrix sharding of the Muon step across GPUs.

The reference is single-process (its README disclaims distributed curvature
synchronisation); its only distributed hint is the ``state_layout()`` tag
marking the momentum buffer "shardable" (``pytorch_opt/optim/muon.py:46-49``).
Here every matrix is an independent unit of work:

* ``lpt_assign`` gives each rank a set of matrices by greedy longest-
  processing-time over their Newton–Schulz FLOPs;
* ``ShardLayout`` places the parameters in one flat buffer: each rank's
  matrices are cut into a few exchange chunks (runs of about equal FLOPs)
  and grouped by shape inside a chunk, so that every shape group is one
  ``[count, rows, cols]`` view, and the buffer is ``[chunk][rank][len]``;
* ``ShardedMuon.step`` updates the local matrices chunk by chunk with the
  grouped kernels and starts each chunk's ``all_gather_into_tensor`` (in
  place: the rank's chunk part is the input, the chunk's slice of the buffer
  the output) as soon as that chunk is stepped, so the exchange of chunk c
  overlaps the Newton–Schulz work of the later chunks. After the step every
  rank holds every updated matrix. Nothing else crosses GPUs.

The same code runs over ``gloo`` on CPU tensors for the host-side tests
(``compute`` can be replaced there, as the kernels need a GPU).
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .muon import MuonGroup, muon_group_step, muon_scale, ns_launches, ns_step_groups, ns_workspace_bytes


def ns_flops(rows: int, cols: int, steps: int = 5) -> float:
    """Dense Newton–Schulz FLOPs of one matrix: steps * (4 m^2 n + 2 m^3), m = min dim."""
    m, n = min(rows, cols), max(rows, cols)
    return float(steps) * (4.0 * m * m * n + 2.0 * m ** 3)


def ns_executed_flops(rows: int, cols: int, steps: int = 5) -> float:
    """FLOPs the tensor cores execute for one matrix under the library's
    schedule (``ns_step_groups``): symmetric m x m results count their lower
    tiles only (256-wide tiles from m = 512, else 128), the full-matrix Gram
    and update count once per step group."""
    m, n = min(rows, cols), max(rows, cols)
    t = 256 if m >= 512 else 128
    k = -(-m // t)
    tri = (k * (k + 1) / 2) / (k * k)
    gram, small, update = 2.0 * m * m * n * tri, 2.0 * m ** 3 * tri, 2.0 * m * m * n
    total = 0.0
    for g in ns_step_groups(rows, cols, steps):
        total += gram + update + (g + 3 * (g - 1)) * small
    return total


def lpt_assign(costs: list[float], world: int) -> list[list[int]]:
    """Greedy LPT: matrices in decreasing cost, each to the least-loaded rank.

    Deterministic (ties broken by index), so every rank computes the same plan.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return out


@dataclass
class _Group:
    shape: tuple[int, int]
    indices: list[int]  # global matrix indices, in slot order
    offset: int         # element offset of the group inside its rank's slot (chunk after chunk)
    chunk: int = 0      # exchange chunk the group belongs to
    flat: int = 0       # element offset of the group in the flat buffer


def chunk_shares(chunks: int) -> list[float]:
    """FLOP share of each exchange chunk, decreasing (e.g. 4: 0.40, 0.30, 0.22,
    0.08): the last chunk's all-gather cannot overlap anything, so it is kept
    small, while each earlier chunk's gather hides behind the larger compute
    of the chunks after it."""
    if chunks <= 1:
        return [1.0]
    w = [float(chunks - c) for c in range(chunks)]
    w[-1] *= 0.5
    t = sum(w)
    return [x / t for x in w]


def bytes_per_flop(rows: int, cols: int) -> float:
    """Exchanged bytes (bf16) per executed Newton–Schulz FLOP of a matrix."""
    return 2.0 * rows * cols / ns_executed_flops(rows, cols)


# Pinned host-to-device copy rate over the fused Muon step's rate of executed
# FLOPs on one B200 (about 50 GB/s against about 1.0 PFLOP/s executed): a
# batch whose gradient bytes per executed NS FLOP exceed this copies longer
# than it computes.
H2D_BYTES_PER_FLOP = 50e9 / 1.0e15


def host_copy_jobs(chunks: list, max_batch: int = 32,
                   bytes_per_flop: float = H2D_BYTES_PER_FLOP) -> list[list[tuple[int, int, int]]]:
    """Order and batch sizes in which gradients copied from host memory are stepped.

    ``chunks``: per exchange chunk, ``(k, count, rows, cols, elem_bytes)`` per
    shape group. The copies (one stream) and the steps (another) form a
    two-stage flow shop. Within a chunk the groups follow Johnson's rule:
    groups whose matrices compute longer than they copy first, by increasing
    copy time, then the others by decreasing compute time. Each group is cut
    into batches as an estimate of both streams goes along: a batch is as
    large as the copy stream's lead over the queued compute lets its copy
    land before the step stream needs it (at least 1, at most ``max_batch``
    matrices), so the step opens with one matrix and the batches grow
    geometrically. Returns ``(k, start, stop)`` triples per chunk.
    """
    copy_end = compute_end = 0.0
    out = []
    for groups in chunks:
        per = []
        for k, count, rows, cols, es in groups:
            a = float(rows * cols * es)
            b = ns_executed_flops(rows, cols) * bytes_per_flop
            per.append((k, count, a, b))
        order = sorted((g for g in per if g[2] < g[3]), key=lambda g: (g[2], g[0])) + \
            sorted((g for g in per if g[2] >= g[3]), key=lambda g: (-g[3], g[0]))
        jobs = []
        for k, count, a, b in order:
            start = 0
            while start < count:
                n = int((compute_end - copy_end) // a) if compute_end > copy_end else 0
                n = max(1, min(max_batch, count - start, n))
                copy_end += n * a
                compute_end = max(compute_end, copy_end) + n * b
                jobs.append((k, start, start + n))
                start += n
        out.append(jobs)
    return out


class ShardLayout:
    """Placement of matrices in a flat parameter buffer, sharded by rank and chunk.

    Each rank's matrices (LPT plan) are processed in decreasing order of
    exchanged bytes per FLOP (Llama: k/v, then gate/up/down, then q/o) and cut
    into ``chunks`` runs whose FLOP shares decrease (``chunk_shares``), so the
    last chunk — whose all-gather is exposed — is small and made of the
    matrices with the fewest bytes per FLOP; inside a run they are grouped by
    shape. The flat buffer is ``[chunk][world][chunk_len[chunk]]``:
    chunk c of every rank sits side by side, so chunk c's exchange is one
    ``all_gather_into_tensor`` whose output is a contiguous slice of the
    buffer, and it can start as soon as every rank has stepped its chunk c
    while the later chunks are still being computed. A rank's *slot* is its
    ``slot = sum(chunk_len)`` elements, chunk after chunk (the layout of
    host-side gradient slots).
    """

    def __init__(self, shapes: list[tuple[int, int]], world: int, steps: int = 5, align: int = 64,
                 chunks: int | None = None):
        self.shapes = [tuple(s) for s in shapes]
        self.world = world
        # Costs are the FLOPs the kernels execute (grouped steps make far-from-
        # square matrices cheaper than the dense formula says).
        costs = [ns_executed_flops(r, c, steps) for r, c in self.shapes]
        self.assign = lpt_assign(costs, world)
        if chunks is None:
            chunks = 1 if world == 1 else 4
        self.chunks = max(1, int(chunks))
        # Per rank: matrices in processing order (largest shapes first), cut into chunk runs.
        runs: list[list[list[int]]] = []
        edges = []
        acc_share = 0.0
        for sh in chunk_shares(self.chunks):
            acc_share += sh
            edges.append(acc_share)
        for r in range(world):
            mine = sorted(self.assign[r], key=lambda i: (-bytes_per_flop(*self.shapes[i]), self.shapes[i], i))
            total = sum(costs[i] for i in mine)
            parts: list[list[int]] = [[] for _ in range(self.chunks)]
            acc = 0.0
            for i in mine:
                mid = (acc + 0.5 * costs[i]) / total if total > 0 else 0.0  # chunk of the matrix's midpoint
                c = next((k for k, e in enumerate(edges) if mid < e), self.chunks - 1)
                parts[c].append(i)
                acc += costs[i]
            runs.append(parts)
        # Chunk lengths (max over ranks), then absolute placement.
        local: list[list[list[tuple]]] = [[[] for _ in range(self.chunks)] for _ in range(world)]
        self.chunk_len = [align] * self.chunks
        for r in range(world):
            for c in range(self.chunks):
                by_shape: dict[tuple[int, int], list[int]] = {}
                for i in runs[r][c]:
                    by_shape.setdefault(self.shapes[i], []).append(i)
                off = 0
                for shape in sorted(by_shape, key=lambda sh: (-sh[0] * sh[1], sh)):
                    idx = sorted(by_shape[shape])
                    local[r][c].append((shape, idx, off))
                    off += len(idx) * shape[0] * shape[1]
                    off = (off + align - 1) // align * align
                self.chunk_len[c] = max(self.chunk_len[c], off)
        self.chunk_base = []
        base = 0
        for c in range(self.chunks):
            self.chunk_base.append(base)
            base += world * self.chunk_len[c]
        self.slot = sum(self.chunk_len)
        self.groups: list[list[_Group]] = []
        self.offset_of: dict[int, tuple[int, int]] = {}  # matrix -> (rank, element offset in the flat buffer)
        for r in range(world):
            groups = []
            slot_base = 0
            for c in range(self.chunks):
                for shape, idx, off in local[r][c]:
                    flat = self.chunk_base[c] + r * self.chunk_len[c] + off
                    groups.append(_Group(shape, idx, slot_base + off, c, flat))
                    n = shape[0] * shape[1]
                    for k, i in enumerate(idx):
                        self.offset_of[i] = (r, flat + k * n)
                slot_base += self.chunk_len[c]
            self.groups.append(groups)

    @property
    def numel(self) -> int:
        return self.world * self.slot

    def matrix(self, flat: torch.Tensor, i: int) -> torch.Tensor:
        """View of matrix i inside a flat buffer laid out by this plan."""
        _, off = self.offset_of[i]
        r, c = self.shapes[i]
        return flat[off:off + r * c].view(r, c)

    def group_views(self, flat: torch.Tensor, rank: int) -> list[torch.Tensor]:
        """``[count, rows, cols]`` views of rank's shape groups inside ``flat`` (full buffer)."""
        out = []
        for g in self.groups[rank]:
            r, c = g.shape
            n = len(g.indices) * r * c
            out.append(flat[g.flat:g.flat + n].view(len(g.indices), r, c))
        return out

    def chunk_part(self, flat: torch.Tensor, rank: int, chunk: int) -> torch.Tensor:
        """Rank's part of one exchange chunk (the all-gather input)."""
        start = self.chunk_base[chunk] + rank * self.chunk_len[chunk]
        return flat[start:start + self.chunk_len[chunk]]

    def chunk_all(self, flat: torch.Tensor, chunk: int) -> torch.Tensor:
        """All ranks' parts of one exchange chunk (the all-gather output)."""
        start = self.chunk_base[chunk]
        return flat[start:start + self.world * self.chunk_len[chunk]]

    def slot_tensor(self, flat: torch.Tensor, rank: int) -> torch.Tensor:
        """Copy of rank's slot (its chunk parts, in chunk order)."""
        return torch.cat([self.chunk_part(flat, rank, c) for c in range(self.chunks)])

    def load_slot(self, flat: torch.Tensor, rank: int, src: torch.Tensor) -> None:
        """Write a slot-shaped tensor into rank's chunk parts of ``flat``."""
        off = 0
        for c in range(self.chunks):
            n = self.chunk_len[c]
            self.chunk_part(flat, rank, c).copy_(src[off:off + n], non_blocking=True)
            off += n

    def slot_elements(self, rank: int) -> int:
        """Matrix elements (padding excluded) of rank's slot."""
        return sum(len(g.indices) * g.shape[0] * g.shape[1] for g in self.groups[rank])

    def flops(self, rank: int, steps: int = 5) -> float:
        return sum(ns_flops(*self.shapes[i], steps) for i in self.assign[rank])


class ShardedMuon:
    """Muon over matrices sharded by ``ShardLayout``; parameters live in one flat buffer.

    ``params_flat``: ``[layout.numel]`` tensor (every rank holds all matrices);
    ``grads_flat``: same layout, only this rank's slot is read.
    """

    def __init__(self, layout: ShardLayout, params_flat: torch.Tensor, grads_flat: torch.Tensor, rank: int,
                 group=None, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True, ns_steps: int = 5,
                 weight_decay: float = 0.0, lr_adjust: str = "spectral", compute=None):
        self.layout = layout
        self.rank = rank
        self.pg = group
        self.params_flat = params_flat
        self.grads_flat = grads_flat
        self.hp = dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps, weight_decay=weight_decay,
                       lr_adjust=lr_adjust)
        pv = layout.group_views(params_flat, rank)
        gv = layout.group_views(grads_flat, rank)
        self.compute = compute
        if compute is None:
            self.groups = [MuonGroup(p, g) for p, g in zip(pv, gv)]
        else:
            self.groups = list(zip(pv, gv))
        self._sq = torch.zeros(max(len(self.groups), 1), dtype=torch.float64, device=params_flat.device)
        self.h2d_bytes_per_flop = H2D_BYTES_PER_FLOP  # batch sizing of step_from_host (host_copy_jobs)
        self._ws = None
        if compute is None and self.groups:
            need = max(ns_workspace_bytes(*g.params.shape, dtype=g.params.dtype) for g in self.groups)
            self._ws = torch.empty(need, dtype=torch.uint8, device=params_flat.device)

    def _step_group(self, k: int, ns_events: list | None, span: tuple[int, int] | None = None) -> None:
        if self.compute is not None:
            p, g = self.groups[k]
            if span is not None:
                p, g = p[span[0]:span[1]], g[span[0]:span[1]]
            self.compute(p, g)
        else:
            muon_group_step(self.groups[k], sq_sum=self._sq[k], workspace=self._ws, ns_events=ns_events, span=span,
                            **self.hp)

    def _gather_chunk(self, c: int):
        """Start chunk c's all-gather (NCCL orders it after the work already queued on the current stream)."""
        return dist.all_gather_into_tensor(self.layout.chunk_all(self.params_flat, c),
                                           self.layout.chunk_part(self.params_flat, self.rank, c),
                                           group=self.pg, async_op=True)

    def _run(self, jobs_of_chunk, ns_events, before_job=None, tail_events=None) -> None:
        """``jobs_of_chunk(c)``: group indices, or ``(k, start, stop)`` spans of groups, in step order."""
        self._sq.zero_()
        pending = []
        for c in range(self.layout.chunks):
            for job in jobs_of_chunk(c):
                if before_job is not None:
                    before_job(job)
                if isinstance(job, tuple):
                    self._step_group(job[0], ns_events, span=job[1:])
                else:
                    self._step_group(job, ns_events)
            if self.layout.world > 1:
                pending.append(self._gather_chunk(c))
        if tail_events is not None:  # after the last local kernel, before the wait for the last exchange
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record()
        for w in pending:
            w.wait()
        if tail_events is not None:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record()
            tail_events.append((t0, t1))

    def _chunk_groups(self, c: int) -> list[int]:
        return [k for k, g in enumerate(self.layout.groups[self.rank]) if g.chunk == c]

    def local_step(self, ns_events: list | None = None) -> None:
        """Update this rank's matrices in place (no communication)."""
        self._sq.zero_()
        for k in range(len(self.groups)):
            self._step_group(k, ns_events)

    def exchange(self) -> None:
        """All-gather every rank's updated matrices into every rank's parameter buffer."""
        if self.layout.world == 1:
            return
        for w in [self._gather_chunk(c) for c in range(self.layout.chunks)]:
            w.wait()

    def step(self, ns_events: list | None = None, tail_events: list | None = None) -> None:
        """Local update and exchange; chunk c's all-gather overlaps the update of chunks c+1..

        ``tail_events``: optional list; a (start, end) pair of CUDA events is
        appended that brackets the part of the step after this rank's last
        kernel (the wait for the exchange still in flight: the exposed
        communication)."""
        self._run(self._chunk_groups, ns_events, tail_events=tail_events)

    def step_from_host(self, host_slot: torch.Tensor, ns_events: list | None = None) -> None:
        """One step whose gradients arrive from host memory.

        ``host_slot``: this rank's gradient slot (``layout.slot`` elements of
        the gradient dtype, chunk after chunk as ``ShardLayout.slot_tensor``
        lays it out), ideally in pinned memory. The gradients are copied on a
        side stream in batches (``host_copy_jobs``: Johnson's order within each
        exchange chunk, batches sized to the copy stream's lead, the first one
        a single matrix) and each batch is stepped as soon as its copy lands,
        so the copies overlap the Newton–Schulz work of the batches before
        them and only the first matrix's copy is exposed. Results are identical to
        copying the slot and calling ``step``.
        """
        if host_slot.numel() < self.layout.slot:
            raise ValueError(f"host_slot holds {host_slot.numel()} elements, the slot needs {self.layout.slot}")
        groups = self.layout.groups[self.rank]

        def grad_of(k):
            return self.groups[k][1] if self.compute is not None else self.groups[k].grads

        def host_view(k, s, e):
            g = groups[k]
            r, c = g.shape
            return host_slot[g.offset + s * r * c:g.offset + e * r * c].view(e - s, r, c)

        es = host_slot.element_size()
        jobs = dict(enumerate(host_copy_jobs(
            [[(k, len(groups[k].indices), *groups[k].shape, es) for k in self._chunk_groups(c)]
             for c in range(self.layout.chunks)], bytes_per_flop=self.h2d_bytes_per_flop)))
        if self.compute is not None:  # host-side (gloo) path: no streams
            for c in range(self.layout.chunks):
                for k, s, e in jobs[c]:
                    grad_of(k)[s:e].copy_(host_view(k, s, e))
            self._run(jobs.__getitem__, ns_events)
            return
        dev = self.params_flat.device
        main = torch.cuda.current_stream(dev)
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(dev)
        cs = self._copy_stream
        cs.wait_stream(main)  # the previous step has finished reading the gradient buffers
        landed = {}
        with torch.cuda.stream(cs):
            for c in range(self.layout.chunks):
                for job in jobs[c]:
                    k, s, e = job
                    grad_of(k)[s:e].copy_(host_view(k, s, e), non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    landed[job] = ev
        self._run(jobs.__getitem__, ns_events, before_job=lambda job: main.wait_event(landed[job]))

    def launches_per_step(self) -> int:
        """Kernels this library launches per local step (the all-gather is NCCL's)."""
        total = 0
        for g in self.groups:
            count, rows, cols = g.params.shape if self.compute is None else g[0].shape
            total += (-(-count // 32)) * ns_launches(rows, cols, int(self.hp["ns_steps"]))
        return total

    def local_update_sq(self) -> float:
        """Sum over local matrices of eff^2 * sum(O^2) (one host read)."""
        total = 0.0
        sq = self._sq.tolist()
        for k, grp in enumerate(self.layout.groups[self.rank]):
            eff = self.hp["lr"] * muon_scale(*grp.shape, self.hp["lr_adjust"])
            total += sq[k] * eff * eff
        return total


# --------------------------------------------------------------------------
# KFAC factor statistics split across GPUs by row bands of the output.
# --------------------------------------------------------------------------

def kfac_band_bounds(d: int, world: int, align: int = 16) -> list[int]:
    """Row boundaries 0 = r_0 <= ... <= r_world = d of the bands of a d x d factor.

    Band k is the rectangle rows [r_k, r_k+1) x columns [0, r_k+1): its rows of
    the lower triangle plus the upper part of its own diagonal block. The
    boundaries give every band about the same area (r_k+1 - r_k) * r_k+1, the
    work of its product; they are multiples of ``align`` (16 keeps bf16 and
    fp32 column offsets 16-byte aligned).
    """
    if world < 1:
        raise ValueError("world must be >= 1")

    def cut(target: float) -> list[int]:
        out = [0]
        while out[-1] < d and len(out) <= world:
            r0 = out[-1]
            r = r0 + align
            while r < d and (r - r0) * r < target:
                r += align
            out.append(min(r, d))
        return out

    lo, hi = 0.0, float(d) * d
    for _ in range(60):  # smallest band area with which world bands reach d
        mid = 0.5 * (lo + hi)
        if cut(mid)[-1] >= d and len(cut(mid)) <= world + 1:
            hi = mid
        else:
            lo = mid
    out = cut(hi)
    while len(out) < world + 1:
        out.append(d)
    return out


def _band_product(band: torch.Tensor, X: torch.Tensor, r0: int, r1: int, alpha: float, beta: float) -> None:
    """band (rows r0..r1 of F, columns 0..r1) <- alpha X[:, r0:r1]^T X[:, :r1] + beta band, on the tensor cores."""
    from . import _lib
    lib = _lib.load()
    rows, d = X.shape
    code = _lib.DTYPE_CODE[X.dtype]
    M, N = r1 - r0, r1
    nbytes = lib.po_matmul_workspace_bytes(1, M, N, rows, code, 1)
    ws = _lib.workspace(nbytes, X.device)
    # A = X[:, r0:r1] stored [K = rows][M] (trans_a), B = X[:, :r1] stored [K][N]; precision 1:
    # split-bf16 for fp32 X, chunked fp32 accumulation for bf16 X (K = rows is long).
    _lib.check(lib.po_matmul(X.data_ptr() + r0 * X.element_size(), d, rows * d, 1, X.data_ptr(), d, rows * d, 0,
                             band.data_ptr(), band.stride(0), M * band.stride(0), code, 1, 1, M, N, rows,
                             float(alpha), float(beta), ws.data_ptr(), nbytes, _lib.stream_ptr(X.device)),
               "po_matmul")


def band_update_(D: torch.Tensor, F: torch.Tensor, X: torch.Tensor, alpha: float, beta: float, first: bool, r0: int,
                 r1: int, compute=None) -> None:
    """One rank's band of the factor update: rows [r0, r1) x columns [0, r1) of
    ``first ? alpha X^T X : beta F + (1 - beta) alpha X^T X`` written into the
    same rows and columns of ``D`` (d x d fp32, or a band-shaped view whose
    row r0 is its first row when ``D.shape[0] == r1 - r0``)."""
    if r1 <= r0:
        return
    band = D[r0:r1, :r1] if D.shape[0] == F.shape[0] else D[:r1 - r0, :r1]
    if first:
        band.zero_()  # products called with beta = 0 must not see stale values (0 * NaN)
    else:
        band.copy_(F[r0:r1, :r1])
    a_eff = alpha if first else (1.0 - beta) * alpha
    b_eff = 0.0 if first else beta
    (compute or _band_product)(band, X, r0, r1, a_eff, b_eff)


def mirror_lower_(F: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """F <- the symmetric matrix whose lower triangle is D's."""
    return F.copy_(torch.tril(D) + torch.tril(D, -1).mT)


_GATHER_BUFFERS: dict = {}


def sharded_syrk_ema_(F: torch.Tensor, X: torch.Tensor, alpha: float, beta: float, first: bool, rank: int = 0,
                      world: int = 1, group=None, compute=None) -> torch.Tensor:
    """KFAC factor update ``F <- first ? alpha X^T X : beta F + (1 - beta) alpha X^T X`` split across ranks.

    The statistic of ``pytorch_opt/curvature/kron.py:95-113`` for one layer,
    with its d x d output cut into row bands of equal work
    (``kfac_band_bounds``): every rank holds the same ``F`` (fp32) and ``X``
    (rows x d, fp32 or bf16), computes only its band on the tensor cores, the
    bands are exchanged with one ``all_gather_into_tensor`` from a cached
    ``[max band][d]`` band into a cached ``[world][max band][d]`` buffer (each
    rank receives the lower triangle once), and each rank mirrors it into the
    full symmetric ``F``. With
    ``world == 1`` the fused triangular SYRK+EMA kernel does the whole update.
    ``compute(band, X, r0, r1, alpha, beta)`` replaces the tensor-core
    product (host-side tests over gloo).
    """
    if X.dim() != 2 or F.dim() != 2 or F.shape[0] != F.shape[1] or F.shape[0] != X.shape[1]:
        raise RuntimeError("sharded_syrk_ema_: expects X (rows, d) and F (d, d)")
    if F.dtype != torch.float32 or not F.is_contiguous():
        raise RuntimeError("sharded_syrk_ema_: F must be a contiguous fp32 tensor")
    d = F.shape[0]
    if world == 1 and compute is None:
        from . import native
        return native.kron_syrk_ema_(F, X, alpha, beta, first)
    bounds = kfac_band_bounds(d, world)
    r0, r1 = bounds[rank], bounds[rank + 1]
    hmax = max(bounds[k + 1] - bounds[k] for k in range(world))
    Xw = (X if X.dtype in (torch.float32, torch.bfloat16) else X.float()).contiguous()
    key = (F.device, d, world, hmax)
    bufs = _GATHER_BUFFERS.get(key)
    if bufs is None:  # the band (input) and the gathered bands (output), reused across calls
        bufs = _GATHER_BUFFERS[key] = (torch.empty(hmax, d, dtype=torch.float32, device=F.device),
                                       torch.empty(world, hmax, d, dtype=torch.float32, device=F.device))
    mine, buf = bufs
    band_update_(mine, F, Xw, alpha, beta, first, r0, r1, compute)
    if world > 1:
        dist.all_gather_into_tensor(buf.view(-1), mine.view(-1), group=group)
    else:
        buf[0].copy_(mine)
    D = F  # assemble the lower triangle in place, then mirror it
    for k in range(world):
        a, b = bounds[k], bounds[k + 1]
        if b > a:
            D[a:b, :b] = buf[k, :b - a, :b]
    return mirror_lower_(F, D)


def sharded_factor_updates_(updates: list, rank: int = 0, world: int = 1, group=None, compute=None) -> list[int]:
    """Many KFAC factor updates (``kron.py:95-113``) shared by the ranks one
    whole factor at a time.

    ``updates``: list of ``(F, X, alpha, beta, first)`` (F d x d fp32, X rows
    x d), the same list on every rank. The factors are assigned to ranks by
    greedy LPT over their SYRK work (rows * d^2); each rank runs the fused
    triangular SYRK+EMA kernel on its own factors, and every factor is then
    broadcast from its owner (NCCL over NVLink), so all ranks end with every
    updated factor. Returns the owner of each update. Unlike the row-band
    split (``sharded_syrk_ema_``), no factor is cut, so each update keeps the
    fused kernel's efficiency; it needs at least as many factors as ranks to
    use every GPU (config 4: A and G on two ranks). ``compute(F, X, alpha,
    beta, first)`` replaces the kernel (host-side tests over gloo).
    """
    if compute is None:
        from . import native
        compute = native.kron_syrk_ema_
    costs = [float(X.shape[0]) * F.shape[0] ** 2 for F, X, *_ in updates]
    owners = [0] * len(updates)
    for r, items in enumerate(lpt_assign(costs, world)):
        for i in items:
            owners[i] = r
    for i, (F, X, alpha, beta, first) in enumerate(updates):
        if owners[i] == rank:
            compute(F, X, alpha, beta, first)
    if world > 1:
        for i, (F, *_rest) in enumerate(updates):
            dist.broadcast(F, src=owners[i], group=group)
    return owners
