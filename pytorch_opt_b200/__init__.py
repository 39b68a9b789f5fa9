"""pytorch_opt_b200 — B200-native (sm_100a) numerics behind ``pytorch_opt.ops``.

Hand-written tcgen05/TMA kernels in ``libpytorch_opt_b200.so`` (C ABI:
``include/pytorch_opt_b200.h``) for the dense-matrix numerics shared by the
Muon, Shampoo, SOAP and KFAC optimizers of pytorch-opt:

* ``native``  — the reference's native-module surface (drop-in for
  ``pytorch_opt.ops.native_build.load()``), plus KFAC and batched extras;
* ``ops``     — the ``pytorch_opt.ops`` public API mirrored on that library;
* ``muon``    — grouped multi-matrix Muon step (momentum, Newton–Schulz, update);
* ``dist``    — FLOP-balanced sharding of matrices over ranks and the NCCL
  all-gather of their updates.
"""

from . import ops, native  # noqa: F401

__version__ = "0.1.0"
