"""Grouped Muon step on the B200 kernels.

The reference updates one matrix at a time (``pytorch_opt/optim/muon.py:70-98``):
momentum, Nesterov, Newton–Schulz, spectral scale, weight decay, update, and a
host sync per matrix for the ``update_rms`` diagnostic (:92). Here matrices
of equal shape live in one ``[count, rows, cols]`` tensor and are stepped
together by ``po_muon_step``: per call of up to 32 matrices, one momentum
pass that also sums each matrix's squared norm, one tiny scale kernel and
the 15 tensor-core products of five Newton–Schulz steps, the last of which
updates the parameters in its epilogue; the diagnostic's sum of squares
accumulates on the device.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch

from . import _lib

_LR_ADJUST = ("spectral", "match_rms_adam", "none")


def muon_scale(rows: int, cols: int, lr_adjust: str = "spectral") -> float:
    """Update scale of ``pytorch_opt/optim/muon.py:51-58``."""
    if lr_adjust == "spectral":
        return max(1.0, rows / cols) ** 0.5
    if lr_adjust == "match_rms_adam":
        return 0.2 * max(rows, cols) ** 0.5
    if lr_adjust == "none":
        return 1.0
    raise ValueError(f"lr_adjust must be one of {_LR_ADJUST}, got {lr_adjust!r}")


@dataclass
class MuonGroup:
    """Same-shape matrix parameters stored together.

    ``params``/``grads``/``momentum``: contiguous ``[count, rows, cols]``
    tensors of one dtype (bf16 or fp32) on one CUDA device.
    """

    params: torch.Tensor
    grads: torch.Tensor
    momentum: torch.Tensor = None
    keep_update: bool = False  # also store the orthogonalised update O in ``_u`` (tests, diagnostics)
    _u: torch.Tensor = field(default=None, repr=False)
    _ws: torch.Tensor = field(default=None, repr=False)

    def __post_init__(self):
        if self.params.dim() != 3 or self.params.shape != self.grads.shape:
            raise ValueError("MuonGroup expects [count, rows, cols] params and grads of the same shape")
        if self.params.dtype not in (torch.bfloat16, torch.float32) or self.grads.dtype != self.params.dtype:
            raise ValueError("MuonGroup params and grads must share dtype bf16 or fp32")
        if not (self.params.is_cuda and self.grads.is_cuda):
            raise RuntimeError("MuonGroup tensors must be on a CUDA device")
        if not (self.params.is_contiguous() and self.grads.is_contiguous()):
            raise ValueError("MuonGroup tensors must be contiguous")
        if self.momentum is None:
            self.momentum = torch.zeros_like(self.params)


def ns_step_groups(rows: int, cols: int, steps: int) -> list[int]:
    """Step groups of the library's Newton-Schulz schedule (bf16 products):
    matrices with min dim m >= 256 and max dim >= 2m run their steps in groups
    of up to three (one Gram and one update of the full matrix per group),
    unless PO_NS_GROUP=0; every other matrix one step at a time."""
    m, n = min(rows, cols), max(rows, cols)
    if steps <= 0:
        return []
    if m < 256 or n < 2 * m or os.environ.get("PO_NS_GROUP", "1") == "0":
        return [1] * steps
    groups, left = [], steps
    while left > 0:
        groups.append(min(3, left))
        left -= groups[-1]
    return groups


def ns_launches(rows: int, cols: int, steps: int) -> int:
    """Kernels one fused Muon call launches: the momentum pass, the scale
    kernel and the products (a group of g >= 2 steps: one Gram, one update,
    g squares and 3 (g - 1) products of m x m matrices; a single step: 3)."""
    return 2 + sum(3 if g == 1 else 2 + g + 3 * (g - 1) for g in ns_step_groups(rows, cols, steps))


def ns_workspace_bytes(count: int, rows: int, cols: int, max_batch: int = 32, dtype=torch.bfloat16) -> int:
    """Workspace one ``muon_group_step`` call needs (fused steps of up to ``max_batch`` matrices)."""
    return int(_lib.load().po_muon_step_workspace_bytes(min(count, max_batch), rows, cols, _lib.DTYPE_CODE[dtype]))


def muon_group_step(group: MuonGroup, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True,
                    ns_steps: int = 5, weight_decay: float = 0.0, lr_adjust: str = "spectral",
                    sq_sum: torch.Tensor | None = None, coeffs=(3.4445, -4.7750, 2.0315), eps: float = 1e-7,
                    workspace: torch.Tensor | None = None, max_batch: int = 32, ns_events: list | None = None,
                    span: tuple[int, int] | None = None) -> None:
    """One Muon update of every matrix in ``group`` (in place).

    ``sq_sum``: optional fp64 CUDA scalar; receives ``sum(O^2)`` of the
    orthogonalised updates (the reference's ``update_rms`` numerator before
    the ``eff^2`` factor). ``workspace``: optional uint8 CUDA buffer of at
    least ``ns_workspace_bytes`` (shared between groups stepped on one
    stream); the fused step runs on at most ``max_batch`` matrices per call to
    bound it. ``ns_events``: optional list; a (start, end) pair of CUDA events
    recorded around the group's fused steps is appended (for timing).
    ``span``: optional ``(start, stop)``; only matrices ``start..stop-1`` of
    the group are updated (their results do not depend on the split).
    """
    lib = _lib.load()
    p = group.params
    count, rows, cols = p.shape
    if p.numel() == 0:
        return
    dev = p.device
    code = _lib.DTYPE_CODE[p.dtype]
    stream = _lib.stream_ptr(dev)
    nb = min(count, max_batch)
    nbytes = lib.po_muon_step_workspace_bytes(nb, rows, cols, code)
    if workspace is None:
        if group._ws is None or group._ws.numel() < nbytes:
            group._ws = _lib.workspace(nbytes, dev)
        workspace = group._ws
    elif workspace.numel() < nbytes:
        raise ValueError(f"workspace too small: {workspace.numel()} < {nbytes} bytes")
    if group.keep_update and group._u is None:
        group._u = torch.empty_like(p)
    mat = rows * cols
    es = p.element_size()
    a, b, c = coeffs
    eff = lr * muon_scale(rows, cols, lr_adjust)
    decay = 1.0 - lr * weight_decay if weight_decay else 1.0
    sq_ptr = sq_sum.data_ptr() if sq_sum is not None else None
    # Measurement switch: PO_MUON_FUSED=0 runs the unfused calls (momentum,
    # Newton-Schulz on a packed copy, update) for A/B timing of the fused step.
    unfused = os.environ.get("PO_MUON_FUSED", "1") == "0"
    first, stop = (0, count) if span is None else (int(span[0]), int(span[1]))
    if not 0 <= first <= stop <= count:
        raise ValueError(f"span {span} outside the group's {count} matrices")
    if unfused and (first, stop) != (0, count):
        raise ValueError("PO_MUON_FUSED=0 steps whole groups only")
    with torch.cuda.device(dev):
        if ns_events is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        if unfused:
            _unfused_group_step(lib, group, code, stream, workspace, momentum, nesterov, ns_steps, coeffs, eps, eff,
                                decay, sq_ptr, max_batch)
        for start in range(first, stop if not unfused else first, max_batch):
            k = min(max_batch, stop - start)
            off = start * mat * es
            o_ptr = group._u.data_ptr() + off if group.keep_update else None
            _lib.check(lib.po_muon_step(group.grads.data_ptr() + off, group.momentum.data_ptr() + off,
                                        p.data_ptr() + off, code, k, rows, cols, float(momentum),
                                        1 if nesterov else 0, int(ns_steps), float(a), float(b), float(c), float(eps),
                                        float(eff), float(decay), sq_ptr, o_ptr, workspace.data_ptr(),
                                        workspace.numel(), stream), "po_muon_step")
        if ns_events is not None:
            ev1.record()
            ns_events.append((ev0, ev1))


def _unfused_group_step(lib, group, code, stream, workspace, momentum, nesterov, ns_steps, coeffs, eps, eff, decay,
                        sq_ptr, max_batch):
    p = group.params
    count, rows, cols = p.shape
    if group._u is None:
        group._u = torch.empty_like(p)
    u = group._u
    mat = rows * cols
    es = p.element_size()
    a, b, c = coeffs
    _lib.check(lib.po_muon_momentum(group.grads.data_ptr(), group.momentum.data_ptr(), u.data_ptr(), code, p.numel(),
                                    float(momentum), 1 if nesterov else 0, stream), "po_muon_momentum")
    for start in range(0, count, max_batch):
        k = min(max_batch, count - start)
        ptr = u.data_ptr() + start * mat * es
        _lib.check(lib.po_newton_schulz(ptr, code, k, rows, cols, cols, mat, ptr, cols, mat, int(ns_steps), float(a),
                                        float(b), float(c), float(eps), -1, workspace.data_ptr(), workspace.numel(),
                                        stream), "po_newton_schulz")
    _lib.check(lib.po_muon_apply(p.data_ptr(), u.data_ptr(), code, p.numel(), float(eff), float(decay), sq_ptr, stream),
               "po_muon_apply")


class GroupedMuon:
    """Muon over many matrix parameters grouped by shape (all on one device)."""

    def __init__(self, groups: list[MuonGroup], lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True,
                 ns_steps: int = 5, weight_decay: float = 0.0, lr_adjust: str = "spectral"):
        if lr_adjust not in _LR_ADJUST:
            raise ValueError(f"lr_adjust must be one of {_LR_ADJUST}, got {lr_adjust!r}")
        self.groups = groups
        self.hp = dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps, weight_decay=weight_decay,
                       lr_adjust=lr_adjust)
        dev = groups[0].params.device if groups else torch.device("cuda")
        # One fp64 accumulator of sum(O^2) per group (groups differ in eff).
        self._sq = torch.zeros(max(len(groups), 1), dtype=torch.float64, device=dev)
        # Groups run one after another on one stream: they share one workspace.
        need = max((ns_workspace_bytes(*g.params.shape, dtype=g.params.dtype) for g in groups), default=1)
        self._ws = _lib.workspace(need, dev)

    def step(self) -> None:
        self._sq.zero_()
        for i, g in enumerate(self.groups):
            muon_group_step(g, sq_sum=self._sq[i], workspace=self._ws, **self.hp)

    def launches_per_step(self) -> int:
        """Kernels this library launches per ``step()``: per fused call of up to 32
        matrices, the momentum pass, the scale (or packing) kernel and the products."""
        total = 0
        for g in self.groups:
            count, rows, cols = g.params.shape
            total += -(-count // 32) * ns_launches(rows, cols, int(self.hp["ns_steps"]))
        return total

    def update_rms(self) -> float:
        """``update_rms`` of the last step as ``pytorch_opt/optim/muon.py:92,99`` defines it (one host read)."""
        if not self.groups:
            return 0.0
        sq = self._sq.tolist()
        total, n_el = 0.0, 0
        for i, g in enumerate(self.groups):
            _, r, c = g.params.shape
            eff = self.hp["lr"] * muon_scale(r, c, self.hp["lr_adjust"])
            total += sq[i] * eff * eff
            n_el += g.params.numel()
        return (total / max(n_el, 1)) ** 0.5
