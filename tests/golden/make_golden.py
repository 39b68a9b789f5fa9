"""Generate the golden fixtures in this directory from the reference itself.

Run in a checkout where kavinravi/pytorch-opt is importable:

    PYTORCH_OPT_REF=/path/to/pytorch-opt python tests/golden/make_golden.py

It imports the reference package (pure-torch ``pytorch_opt.ops.reference``
backend, ``KronTracker``, ``kfac_factored_damping``, ``KFAC._damped_inverse``
and the ``Muon`` optimizer), runs them on small seeded inputs on the CPU, and
writes inputs and outputs to ``*.npz`` next to this script. The fixtures pin
the numpy oracle in ``oracle/ops_np.py`` (tests/test_oracle_golden.py) and
are the fixed vectors the GPU parity tests compare against.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference():
    root = os.environ.get("PYTORCH_OPT_REF")
    if root is None:
        raise SystemExit("set PYTORCH_OPT_REF to the reference checkout (the directory holding pytorch_opt/)")
    sys.path.insert(0, root)
    import pytorch_opt  # noqa: F401
    from pytorch_opt.ops import reference as R
    from pytorch_opt.curvature.kron import KronTracker
    from pytorch_opt.curvature.damping import kfac_factored_damping
    from pytorch_opt.optim.kfac import KFAC
    from pytorch_opt.optim.muon import Muon
    return R, KronTracker, kfac_factored_damping, KFAC, Muon


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).numpy() if t.dtype != torch.float64 else t.detach().numpy()


def _spd(n, seed, lo=0.5, hi=4.0, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    Q, _ = torch.linalg.qr(torch.randn(n, n, generator=g, dtype=torch.float64))
    lam = torch.linspace(lo, hi, n, dtype=torch.float64)
    return (Q @ torch.diag(lam) @ Q.T).to(dtype)


def make_ns(R) -> dict:
    out = {}
    cases = [
        ((8, 5), torch.float32, 5, 1.0), ((5, 8), torch.float32, 5, 1.0), ((4, 6, 9), torch.float32, 5, 1.0),
        ((16, 32), torch.float32, 5, 1.0), ((32, 64), torch.float64, 5, 1.0), ((24, 40), torch.bfloat16, 5, 0.02),
        ((64, 48), torch.float32, 5, 0.02), ((3, 3), torch.float32, 5, 1.0), ((40, 24), torch.bfloat16, 3, 1.0),
        ((96, 200), torch.float32, 5, 1.0),
    ]
    for i, (shape, dt, steps, scale) in enumerate(cases):
        g = torch.Generator().manual_seed(100 + i)
        G = (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).to(dt)
        O = R.newton_schulz_orthogonalize(G, steps=steps)
        out[f"case{i}_in"] = _f32(G) if dt != torch.float64 else G.numpy()
        out[f"case{i}_out"] = _f32(O) if dt != torch.float64 else O.numpy()
        out[f"case{i}_meta"] = np.array([steps, {torch.float32: 0, torch.bfloat16: 1, torch.float64: 3}[dt]])
    # (semi-)orthogonal inputs map to a scalar multiple (reference test_ops_reference.py:72-80)
    for j, shape in enumerate([(8, 8), (12, 6)]):
        g = torch.Generator().manual_seed(200 + j)
        Q, _ = torch.linalg.qr(torch.randn(*shape, generator=g))
        O = R.newton_schulz_orthogonalize(Q, steps=10)
        k = len(cases) + j
        out[f"case{k}_in"] = Q.numpy()
        out[f"case{k}_out"] = O.numpy()
        out[f"case{k}_meta"] = np.array([10, 0])
    out["ncases"] = np.array(len(cases) + 2)
    return out


def make_roots(R) -> dict:
    out = {}
    cases = []
    A6 = _spd(6, 1)
    for p in (1, 2, 4):
        for method in ("eigh", "newton"):
            cases.append((A6, p, 1e-6, method))
    g = torch.Generator().manual_seed(5)
    B = torch.randn(3, 5, 5, generator=g)
    cases.append(((B @ B.mT + 0.1 * torch.eye(5)).to(torch.float32), 4, 1e-6, "auto"))
    g = torch.Generator().manual_seed(6)
    Gm = torch.randn(32, 64, generator=g)
    cases.append(((Gm @ Gm.T / 64 + 1e-6 * torch.eye(32)).to(torch.float32), 4, 1e-8, "newton"))
    cases.append((_spd(12, 7, 0.2, 3.0).to(torch.float32), 3, 0.0, "newton"))
    g = torch.Generator().manual_seed(8)
    Gm = torch.randn(48, 96, generator=g)
    cases.append(((Gm @ Gm.T / 96).to(torch.float32), 1, 1e-3, "newton"))
    cases.append((_spd(8, 9), 2, 0.37, "newton"))
    for i, (A, p, damping, method) in enumerate(cases):
        X = R.inverse_matrix_root(A, p, damping=damping, method=method)
        out[f"case{i}_in"] = A.numpy()
        out[f"case{i}_out"] = X.numpy()
        out[f"case{i}_meta"] = np.array([p, damping, ("auto", "eigh", "newton").index(method)], dtype=np.float64)
    out["ncases"] = np.array(len(cases))
    return out


def make_kron(R) -> dict:
    out = {}
    for i, (m, n) in enumerate([(4, 7), (16, 24), (33, 17)]):
        g = torch.Generator().manual_seed(12 + i)
        G1, G2 = (torch.randn(m, n, generator=g) for _ in range(2))
        out[f"case{i}_G1"] = G1.numpy()
        out[f"case{i}_G2"] = G2.numpy()
        for beta in (1.0, 0.9):
            L = torch.zeros(m, m)
            Rr = torch.zeros(n, n)
            R.kron_factor_update_(L, Rr, G1, beta2=beta)
            R.kron_factor_update_(L, Rr, G2, beta2=beta)
            out[f"case{i}_L_{beta}"] = L.numpy()
            out[f"case{i}_R_{beta}"] = Rr.numpy()
    out["ncases"] = np.array(3)
    return out


def make_precond(R) -> dict:
    out = {}
    for i, (m, n) in enumerate([(4, 7), (9, 5), (16, 16)]):
        g = torch.Generator().manual_seed(30 + i)
        Lr, G, Rr = torch.randn(m, m, generator=g), torch.randn(m, n, generator=g), torch.randn(n, n, generator=g)
        out[f"case{i}_L"], out[f"case{i}_G"], out[f"case{i}_R"] = Lr.numpy(), G.numpy(), Rr.numpy()
        out[f"case{i}_out"] = R.precond_apply_two_sided(Lr, G, Rr).numpy()
    out["ncases"] = np.array(3)
    return out


def make_kfac(KronTracker, kfac_factored_damping, KFAC) -> dict:
    out = {}
    for i, (bias, ema) in enumerate([(False, 0.95), (True, 0.95), (False, None)]):
        torch.manual_seed(40 + i)
        model = torch.nn.Sequential(torch.nn.Linear(6, 5, bias=bias))
        lin = model[0]
        tr = KronTracker(model, ema_decay=ema)
        tr.enabled = True
        g = torch.Generator().manual_seed(50 + i)
        for step in range(3):
            a = torch.randn(7, 6, generator=g)
            go = torch.randn(7, 5, generator=g) * 0.1
            tr._on_grad_out(lin, a, go)
            out[f"case{i}_a{step}"] = a.numpy()
            out[f"case{i}_g{step}"] = go.numpy()
        name = tr._module_names[lin]
        A, G = tr.factors[name]["A"], tr.factors[name]["G"]
        out[f"case{i}_A"], out[f"case{i}_G"] = A.numpy(), G.numpy()
        ga, gg = kfac_factored_damping(A, G, 1e-3)
        out[f"case{i}_gammas"] = np.array([ga, gg])
        iA, cA = KFAC._damped_inverse(A, ga)
        iG, cG = KFAC._damped_inverse(G, gg)
        out[f"case{i}_iA"], out[f"case{i}_iG"] = iA.numpy(), iG.numpy()
        out[f"case{i}_conds"] = np.array([cA, cG])
        out[f"case{i}_meta"] = np.array([1.0 if bias else 0.0, -1.0 if ema is None else ema])
    out["ncases"] = np.array(3)
    return out


def make_muon(Muon) -> dict:
    out = {}
    torch.manual_seed(60)
    shapes = [(32, 48), (48, 32), (16, 16)]
    params = [torch.nn.Parameter((torch.randn(*s) * 0.05).to(torch.bfloat16)) for s in shapes]
    for k, p in enumerate(params):
        out[f"p{k}_init"] = _f32(p.data)
    opt = Muon(params, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5, weight_decay=0.01)
    g = torch.Generator().manual_seed(61)
    for step in range(2):
        for k, p in enumerate(params):
            p.grad = (torch.randn(*p.shape, generator=g) * 0.02).to(torch.bfloat16)
            out[f"p{k}_grad{step}"] = _f32(p.grad)
        opt.step()
        out[f"update_rms{step}"] = np.array(opt.diagnostics["update_rms"])
    for k, p in enumerate(params):
        out[f"p{k}_final"] = _f32(p.data)
        out[f"p{k}_buf"] = _f32(opt.state[p]["momentum_buffer"])
    out["nparams"] = np.array(len(shapes))
    out["hparams"] = np.array([0.02, 0.95, 1.0, 5.0, 0.01])
    return out


def make_ekfac() -> dict:
    """EKFAC._precondition (optim/ekfac.py:44-58) on two consecutive gradients.

    The method is called unbound on a stand-in holding exactly the state it
    reads (eigenbases, damping, running scales, decay), so no model or hooks
    are needed; eigenbases come from fp64 eigh of SPD factors, as in
    ``_refresh_inverses`` (:27-42).
    """
    from types import SimpleNamespace
    from pytorch_opt.optim.ekfac import EKFAC
    out = {}
    cases = [(48, 80, 0.95, 1e-3), (96, 33, 0.9, 1e-2)]
    for i, (m, n, decay, lam) in enumerate(cases):
        _, QG = torch.linalg.eigh(_spd(m, 300 + i))
        _, QA = torch.linalg.eigh(_spd(n, 400 + i))
        QG, QA = QG.to(torch.float32), QA.to(torch.float32)
        me = SimpleNamespace(_inv={"w": {"QG": QG, "QA": QA}}, param_groups=[{"damping": lam}], _scales={},
                             _scale_decay=decay)
        g = torch.Generator().manual_seed(500 + i)
        V1 = torch.randn(m, n, generator=g)
        V2 = torch.randn(m, n, generator=g)
        o1 = EKFAC._precondition(me, "w", V1)
        s1 = me._scales["w"].clone()
        o2 = EKFAC._precondition(me, "w", V2)
        s2 = me._scales["w"].clone()
        out.update({f"case{i}_QG": _f32(QG), f"case{i}_QA": _f32(QA), f"case{i}_V1": _f32(V1),
                    f"case{i}_V2": _f32(V2), f"case{i}_out1": _f32(o1), f"case{i}_out2": _f32(o2),
                    f"case{i}_s1": _f32(s1), f"case{i}_s2": _f32(s2),
                    f"case{i}_hp": np.array([decay, lam], dtype=np.float64)})
    out["ncases"] = np.array(len(cases))
    return out


def make_soap() -> dict:
    """SOAP.step (optim/soap.py:66-131) on one fp32 matrix with a basis
    refresh every step (precondition_frequency=1): the state after each of
    three steps and the gradient of the next, so that a refresh's transport
    (:101-108) can be checked from the state before and after it."""
    from pytorch_opt.optim import SOAP
    out = {}
    m, n = 24, 40
    g = torch.Generator().manual_seed(600)
    p = torch.nn.Parameter(torch.randn(m, n, generator=g))
    opt = SOAP([p], lr=3e-3, precondition_frequency=1)
    grads = [torch.randn(m, n, generator=g) * 0.1 for _ in range(3)]
    for k, gr in enumerate(grads):
        p.grad = gr.clone()
        opt.step()
        st = opt.state[p]
        snap = {"grad": gr, "L": st["L"], "R": st["R"], "QL": st["Q_L"], "QR": st["Q_R"], "V": st["exp_avg_sq"],
                "p": p.detach()}
        out.update({f"step{k}_{key}": _f32(t.clone()) for key, t in snap.items()})  # copies: the state is updated in place
    out["hp"] = np.array([opt.param_groups[0]["betas"][1], opt.param_groups[0]["shampoo_beta"]], dtype=np.float64)
    out["nsteps"] = np.array(len(grads))
    return out


def main(only=None) -> None:
    """Write every fixture, or only the named ones (e.g. ``ekfac``)."""
    R, KronTracker, kfac_factored_damping, KFAC, Muon = _import_reference()
    torch.set_num_threads(1)
    makers = {
        "ns": lambda: make_ns(R), "roots": lambda: make_roots(R), "kron": lambda: make_kron(R),
        "precond": lambda: make_precond(R),
        "kfac": lambda: make_kfac(KronTracker, kfac_factored_damping, KFAC), "muon": lambda: make_muon(Muon),
        "ekfac": make_ekfac, "soap": make_soap,
    }
    for name, make in makers.items():
        if only and name not in only:
            continue
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **make())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
