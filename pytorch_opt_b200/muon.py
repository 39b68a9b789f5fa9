"""Grouped Muon step on the B200 kernels.

The reference updates one matrix at a time (``pytorch_opt/optim/muon.py:70-98``):
momentum, Nesterov, Newton–Schulz, spectral scale, weight decay, update, and a
host sync per matrix for the ``update_rms`` diagnostic (:92). Here matrices
of equal shape live in one ``[count, rows, cols]`` tensor and are stepped
together: one momentum launch, one batched Newton–Schulz (15 tensor-core
launches for five steps), one update launch per shape group, and the
diagnostic's sum of squares accumulates on the device.
"""

from __future__ import annotations

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


def muon_group_step(group: MuonGroup, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True,
                    ns_steps: int = 5, weight_decay: float = 0.0, lr_adjust: str = "spectral",
                    sq_sum: torch.Tensor | None = None, coeffs=(3.4445, -4.7750, 2.0315), eps: float = 1e-7) -> None:
    """One Muon update of every matrix in ``group`` (in place).

    ``sq_sum``: optional fp64 CUDA scalar; receives ``sum(O^2)`` of the
    orthogonalised updates (the reference's ``update_rms`` numerator before
    the ``eff^2`` factor).
    """
    lib = _lib.load()
    p = group.params
    count, rows, cols = p.shape
    n = p.numel()
    if n == 0:
        return
    dev = p.device
    code = _lib.DTYPE_CODE[p.dtype]
    stream = _lib.stream_ptr(dev)
    if group._u is None:
        group._u = torch.empty_like(p)
    nbytes = lib.po_ns_workspace_bytes(count, rows, cols)
    if group._ws is None or group._ws.numel() < nbytes:
        group._ws = _lib.workspace(nbytes, dev)
    u = group._u
    with torch.cuda.device(dev):
        _lib.check(lib.po_muon_momentum(group.grads.data_ptr(), group.momentum.data_ptr(), u.data_ptr(), code, n,
                                        float(momentum), 1 if nesterov else 0, stream), "po_muon_momentum")
        a, b, c = coeffs
        # The orthogonalised update overwrites u in place: Newton–Schulz reads its
        # input only in the packing pass that precedes every product.
        _lib.check(lib.po_newton_schulz(u.data_ptr(), code, count, rows, cols, cols, rows * cols, u.data_ptr(), cols,
                                        rows * cols, int(ns_steps), float(a), float(b), float(c), float(eps), -1,
                                        group._ws.data_ptr(), nbytes, stream), "po_newton_schulz")
        eff = lr * muon_scale(rows, cols, lr_adjust)
        decay = 1.0 - lr * weight_decay if weight_decay else 1.0
        _lib.check(lib.po_muon_apply(p.data_ptr(), u.data_ptr(), code, n, float(eff), float(decay),
                                     sq_sum.data_ptr() if sq_sum is not None else None, stream), "po_muon_apply")


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

    def step(self) -> None:
        self._sq.zero_()
        for i, g in enumerate(self.groups):
            muon_group_step(g, sq_sum=self._sq[i], **self.hp)

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
