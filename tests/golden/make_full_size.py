"""Generate ``full_size.npz``: the reference's own outputs at the benchmark's
full problem sizes, stored as small two-sided sketches.

Run where kavinravi/pytorch-opt is importable (takes a few minutes on the CPU):

    PYTORCH_OPT_REF=/path/to/pytorch-opt python tests/golden/make_full_size.py [ns] [roots] [kfac]

For each case the reference runs on the CPU on inputs drawn from a seeded
CPU generator (so any machine can redraw them bit for bit):

* Newton–Schulz (``pytorch_opt.ops.reference.newton_schulz_orthogonalize``)
  on the four Llama-3-8B matrix shapes, bf16 0.02 N(0,1) inputs (seed
  1000 + i), 5 steps; as Muon calls it (bf16 in, bf16 out), and on the same
  values in fp32 and in fp64;
* inverse 4th roots (``inverse_matrix_root(..., method="newton")``, fp64) of
  config-3 Shampoo factors L = G G^T / 2d + 1e-6 I (G d x 2d N(0,1), seed
  100 d), damping 1e-8, with the iteration count of the reference's loop
  (counted through its one ``torch.linalg.matrix_power`` call per step);
* KFAC config 4: ``KronTracker`` factors A, G of two 8192 x 4096 bf16
  batches (first call clones, second EMA 0.95), ``kfac_factored_damping``
  with lambda 1e-3, and ``KFAC._damped_inverse`` (fp64 eigh) with its
  condition numbers.

A full output would be hundreds of MB, so each is stored as the 32 x 32
sketch L^T X R (``oracle.ops_torch.two_sided_sketch``) with its seeds.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.ops_torch import two_sided_sketch  # noqa: E402

NS_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]
ROOT_DIMS = [1024, 2048, 4096]
KFAC_ROWS, KFAC_DIM = 8192, 4096


def ns_input(i: int) -> torch.Tensor:
    rows, cols = NS_SHAPES[i]
    g = torch.Generator().manual_seed(1000 + i)
    return (torch.randn(rows, cols, generator=g) * 0.02).bfloat16()


def shampoo_factor(d: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(100 * d)
    G = torch.randn(d, 2 * d, generator=g)
    return G @ G.T / (2 * d) + 1e-6 * torch.eye(d)


def kfac_batch(seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(KFAC_ROWS, KFAC_DIM, generator=g).bfloat16()


def _import_reference():
    root = os.environ.get("PYTORCH_OPT_REF")
    if root is None:
        raise SystemExit("set PYTORCH_OPT_REF to the reference checkout (the directory holding pytorch_opt/)")
    sys.path.insert(0, root)
    from pytorch_opt.ops import reference as R
    from pytorch_opt.curvature.kron import KronTracker
    from pytorch_opt.curvature.damping import kfac_factored_damping
    from pytorch_opt.optim.kfac import KFAC
    return R, KronTracker, kfac_factored_damping, KFAC


def main(only=None) -> None:
    """Write every part (ns, roots, kfac), or only the named ones (the others
    are kept from an existing full_size.npz)."""
    R, KronTracker, kfac_factored_damping, KFAC = _import_reference()
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    path = os.path.join(HERE, "full_size.npz")
    out = dict(np.load(path)) if os.path.exists(path) else {}
    for i, (rows, cols) in enumerate(NS_SHAPES):
        if only and "ns" not in only:
            break
        G = ns_input(i)
        O = R.newton_schulz_orthogonalize(G, steps=5)
        out[f"ns{i}_sketch"] = two_sided_sketch(O, 7000 + i, 8000 + i).numpy()
        # The same values through the fp32 path (fp32 output, no final
        # rounding to bf16). On the CPU its Frobenius norm is summed in fp32
        # and is 0.5 % low at 14336 x 4096, which moves the output by ~5e-3.
        O32 = R.newton_schulz_orthogonalize(G.float(), steps=5)
        out[f"ns{i}_sketch_f32"] = two_sided_sketch(O32, 7000 + i, 8000 + i).numpy()
        # And in fp64 (the reference's work dtype for fp64 input): pins the
        # full-size checker.
        O64 = R.newton_schulz_orthogonalize(G.double(), steps=5)
        out[f"ns{i}_sketch_f64"] = two_sided_sketch(O64, 7000 + i, 8000 + i).numpy()
        out[f"ns{i}_meta"] = np.array([rows, cols, 1000 + i, 7000 + i, 8000 + i])
        print("ns", rows, cols, flush=True)

    real_power = torch.linalg.matrix_power
    for d in ROOT_DIMS:
        if only and "roots" not in only:
            break
        calls = [0]

        def counting_power(M, n, _real=real_power):
            calls[0] += 1
            return _real(M, n)
        torch.linalg.matrix_power = counting_power
        try:
            X = R.inverse_matrix_root(shampoo_factor(d), 4, damping=1e-8, method="newton")
        finally:
            torch.linalg.matrix_power = real_power
        out[f"root{d}_iters"] = np.array(calls[0])
        out[f"root{d}_sketch"] = two_sided_sketch(X, 7100 + d, 8100 + d).numpy()
        print("root", d, calls[0], flush=True)

    if only and "kfac" not in only:
        np.savez_compressed(path, **out)
        print("wrote", path)
        return
    model = torch.nn.Sequential(torch.nn.Linear(KFAC_DIM, KFAC_DIM, bias=False))
    lin = model[0]
    tr = KronTracker(model, ema_decay=0.95)
    tr.enabled = True
    for step, (sa, sg) in enumerate([(1, 2), (3, 4)]):
        tr._on_grad_out(lin, kfac_batch(sa), kfac_batch(sg))
        name = tr._module_names[lin]
        A, G = tr.factors[name]["A"], tr.factors[name]["G"]
        out[f"kfac_A{step}_sketch"] = two_sided_sketch(A, 7200 + step, 8200 + step).numpy()
        out[f"kfac_G{step}_sketch"] = two_sided_sketch(G, 7300 + step, 8300 + step).numpy()
        print("kfac step", step, flush=True)
    ga, gg = kfac_factored_damping(A, G, 1e-3)
    out["kfac_gammas"] = np.array([ga, gg])
    out["kfac_traces"] = np.array([float(A.diagonal().sum()), float(G.diagonal().sum())])
    iA, cA = KFAC._damped_inverse(A, ga)
    out["kfac_iA_sketch"] = two_sided_sketch(iA, 7400, 8400).numpy()
    iG, cG = KFAC._damped_inverse(G, gg)
    out["kfac_iG_sketch"] = two_sided_sketch(iG, 7500, 8500).numpy()
    out["kfac_conds"] = np.array([cA, cG])
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
