"""Per-matrix sharding of the Muon step across GPUs.

The reference is single-process (its README disclaims distributed curvature
synchronisation); its only distributed hint is the ``state_layout()`` tag
marking the momentum buffer "shardable" (``pytorch_opt/optim/muon.py:46-49``).
Here every matrix is an independent unit of work:

* ``lpt_assign`` gives each rank a set of matrices by greedy longest-
  processing-time over their Newton–Schulz FLOPs;
* ``ShardLayout`` places the parameters in one flat buffer of
  ``world * slot`` elements, rank r's matrices packed (grouped by shape) in
  slot r, so that every shape group is one ``[count, rows, cols]`` view;
* ``ShardedMuon.step`` updates the local slot with the grouped kernels and
  then runs one ``all_gather_into_tensor`` whose output is the parameter
  buffer itself (in place: the local slot is the input), so after the step
  every rank holds every updated matrix. Nothing else crosses GPUs.

The same code runs over ``gloo`` on CPU tensors for the host-side tests
(``compute`` can be replaced there, as the kernels need a GPU).
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .muon import MuonGroup, muon_group_step, muon_scale, ns_workspace_bytes


def ns_flops(rows: int, cols: int, steps: int = 5) -> float:
    """Dense Newton–Schulz FLOPs of one matrix: steps * (4 m^2 n + 2 m^3), m = min dim."""
    m, n = min(rows, cols), max(rows, cols)
    return float(steps) * (4.0 * m * m * n + 2.0 * m ** 3)


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
    offset: int         # element offset of the group inside its rank's slot


class ShardLayout:
    """Placement of matrices in a flat ``[world * slot]`` buffer (slot r = rank r's matrices)."""

    def __init__(self, shapes: list[tuple[int, int]], world: int, steps: int = 5, align: int = 64):
        self.shapes = [tuple(s) for s in shapes]
        self.world = world
        self.assign = lpt_assign([ns_flops(r, c, steps) for r, c in self.shapes], world)
        self.groups: list[list[_Group]] = []
        self.offset_of: dict[int, tuple[int, int]] = {}  # matrix -> (rank, element offset in the flat buffer)
        slot = 0
        per_rank = []
        for r in range(world):
            by_shape: dict[tuple[int, int], list[int]] = {}
            for i in sorted(self.assign[r]):
                by_shape.setdefault(self.shapes[i], []).append(i)
            groups, off = [], 0
            for shape in sorted(by_shape, key=lambda s: (-s[0] * s[1], s)):
                idx = by_shape[shape]
                groups.append(_Group(shape, idx, off))
                off += len(idx) * shape[0] * shape[1]
                off = (off + align - 1) // align * align
            per_rank.append((groups, off))
            slot = max(slot, off)
        self.slot = max(slot, align)
        for r, (groups, _) in enumerate(per_rank):
            self.groups.append(groups)
            for g in groups:
                n = g.shape[0] * g.shape[1]
                for k, i in enumerate(g.indices):
                    self.offset_of[i] = (r, r * self.slot + g.offset + k * n)

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
        base = rank * self.slot
        out = []
        for g in self.groups[rank]:
            r, c = g.shape
            n = len(g.indices) * r * c
            out.append(flat[base + g.offset: base + g.offset + n].view(len(g.indices), r, c))
        return out

    def slot_view(self, flat: torch.Tensor, rank: int) -> torch.Tensor:
        return flat[rank * self.slot:(rank + 1) * self.slot]

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
        self._ws = None
        if compute is None and self.groups:
            need = max(ns_workspace_bytes(*g.params.shape) for g in self.groups)
            self._ws = torch.empty(need, dtype=torch.uint8, device=params_flat.device)

    def local_step(self, ns_events: list | None = None) -> None:
        """Update this rank's matrices in place (no communication)."""
        self._sq.zero_()
        if self.compute is not None:
            for p, g in self.groups:
                self.compute(p, g)
            return
        for i, g in enumerate(self.groups):
            muon_group_step(g, sq_sum=self._sq[i], workspace=self._ws, ns_events=ns_events, **self.hp)

    def exchange(self) -> None:
        """All-gather every rank's updated slot into every rank's parameter buffer."""
        if self.layout.world == 1:
            return
        local = self.layout.slot_view(self.params_flat, self.rank)
        dist.all_gather_into_tensor(self.params_flat, local, group=self.pg)

    def step(self, ns_events: list | None = None) -> None:
        self.local_step(ns_events)
        self.exchange()

    def step_from_host(self, host_slot: torch.Tensor, ns_events: list | None = None) -> None:
        """One step whose gradients arrive from host memory.

        ``host_slot``: this rank's gradient slot (``layout.slot`` elements of
        the gradient dtype), ideally in pinned memory. Each shape group's
        gradients are copied on a side stream, smallest group first, and the
        group is stepped as soon as its copy lands, so the copies of the later
        groups overlap the Newton–Schulz work of the earlier ones; only the
        first (smallest) copy is exposed. Results are identical to copying the
        whole slot and calling ``step``.
        """
        if host_slot.numel() < self.layout.slot:
            raise ValueError(f"host_slot holds {host_slot.numel()} elements, the slot needs {self.layout.slot}")
        groups = self.layout.groups[self.rank]

        def host_view(k):
            g = groups[k]
            r, c = g.shape
            return host_slot[g.offset:g.offset + len(g.indices) * r * c].view(len(g.indices), r, c)

        if self.compute is not None:  # host-side (gloo) path: no streams
            for k, (_, grad) in enumerate(self.groups):
                grad.copy_(host_view(k))
            self.step(ns_events)
            return
        dev = self.params_flat.device
        main = torch.cuda.current_stream(dev)
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(dev)
        cs = self._copy_stream
        order = sorted(range(len(self.groups)), key=lambda k: (self.groups[k].grads.numel(), k))
        cs.wait_stream(main)  # the previous step has finished reading the gradient buffers
        landed = []
        with torch.cuda.stream(cs):
            for k in order:
                self.groups[k].grads.copy_(host_view(k), non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                landed.append(ev)
        self._sq.zero_()
        for k, ev in zip(order, landed):
            main.wait_event(ev)
            muon_group_step(self.groups[k], sq_sum=self._sq[k], workspace=self._ws, ns_events=ns_events, **self.hp)
        self.exchange()

    def launches_per_step(self) -> int:
        """Kernels this library launches per local step (the all-gather is NCCL's)."""
        total = 0
        for g in self.groups:
            count = g.params.shape[0] if self.compute is None else g[0].shape[0]
            total += 2 + (-(-count // 32)) * (2 + 3 * int(self.hp["ns_steps"]))
        return total

    def local_update_sq(self) -> float:
        """Sum over local matrices of eff^2 * sum(O^2) (one host read)."""
        total = 0.0
        sq = self._sq.tolist()
        for k, grp in enumerate(self.layout.groups[self.rank]):
            eff = self.hp["lr"] * muon_scale(*grp.shape, self.hp["lr_adjust"])
            total += sq[k] * eff * eff
        return total
