"""ctypes binding of the C ABI in ``include/pytorch_opt_b200.h``.

The shared library is built in-tree by ``pytorch_opt_b200.build``. Loading
fails loudly: there is no CPU or library fallback behind these entry points.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libpytorch_opt_b200.so")

# dtype codes of the C ABI
PO_F32, PO_BF16, PO_F16, PO_F64 = 0, 1, 2, 3
DTYPE_CODE = {torch.float32: PO_F32, torch.bfloat16: PO_BF16, torch.float16: PO_F16, torch.float64: PO_F64}

_vp, _i, _ll, _f, _d, _sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_double,
                            ctypes.c_size_t)

# name -> (restype, argtypes); mirrors include/pytorch_opt_b200.h
SIGNATURES = {
    "po_last_error": (ctypes.c_char_p, []),
    "po_device_error": (_i, [_i]),
    "po_version": (ctypes.c_char_p, []),
    "po_selftest_wait_timeout": (_i, [ctypes.c_ulonglong, _i, _vp]),
    "po_gemm_profile": (_i, [_i, _vp, _i]),
    "po_ns_workspace_bytes": (_sz, [_ll, _ll, _ll]),
    "po_newton_schulz": (_i, [_vp, _i, _ll, _ll, _ll, _ll, _ll, _vp, _ll, _ll, _i, _f, _f, _f, _f, _i, _vp, _sz,
                              _vp]),
    "po_newton_schulz_static": (_i, [_vp, _i, _ll, _ll, _ll, _ll, _ll, _vp, _ll, _ll, _i, _f, _f, _f, _f, _i,
                                     _vp]),
    "po_root_workspace_bytes": (_sz, [_ll, _ll, _i]),
    "po_inverse_root": (_i, [_vp, _i, _ll, _ll, _ll, _ll, _vp, _ll, _ll, _i, _d, _i, _d, _vp, _vp, _sz, _vp]),
    "po_kron_workspace_bytes": (_sz, [_ll, _ll, _i]),
    "po_kron_factor_update": (_i, [_vp, _ll, _vp, _ll, _vp, _i, _ll, _ll, _ll, _d, _vp, _sz, _vp]),
    "po_syrk_workspace_bytes": (_sz, [_ll, _ll, _i]),
    "po_syrk_ema": (_i, [_vp, _ll, _ll, _vp, _i, _ll, _ll, _d, _d, _i, _vp, _vp, _sz, _vp]),
    "po_precond_workspace_bytes": (_sz, [_ll, _ll, _i]),
    "po_precond_apply": (_i, [_vp, _ll, _vp, _ll, _vp, _ll, _vp, _ll, _i, _ll, _ll, _vp, _sz, _vp]),
    "po_precond_apply_norm": (_i, [_vp, _ll, _vp, _ll, _vp, _ll, _vp, _ll, _i, _ll, _ll, _vp, _vp, _sz, _vp]),
    "po_precond_apply_ex": (_i, [_vp, _ll, _i, _vp, _ll, _vp, _ll, _i, _vp, _ll, _i, _ll, _ll, _vp, _vp, _sz, _vp]),
    "po_soap_transport_workspace_bytes": (_sz, [_ll, _ll, _i]),
    "po_soap_transport": (_i, [_vp, _vp, _ll, _vp, _vp, _ll, _vp, _ll, _i, _ll, _ll, _vp, _sz, _vp]),
    "po_ekfac_workspace_bytes": (_sz, [_ll, _ll]),
    "po_ekfac_precondition": (_i, [_vp, _ll, _vp, _ll, _vp, _ll, _vp, _ll, _vp, _ll, _ll, _ll, _i, _f, _f, _vp, _sz,
                                   _vp]),
    "po_muon_momentum": (_i, [_vp, _vp, _vp, _i, _ll, _f, _i, _vp]),
    "po_muon_apply": (_i, [_vp, _vp, _i, _ll, _f, _f, _vp, _vp]),
    "po_muon_step_workspace_bytes": (_sz, [_ll, _ll, _ll, _i]),
    "po_muon_step": (_i, [_vp, _vp, _vp, _i, _ll, _ll, _ll, _f, _i, _i, _f, _f, _f, _f, _f, _f, _vp, _vp, _vp, _sz,
                          _vp]),
    "po_matmul_workspace_bytes": (_sz, [_ll, _ll, _ll, _ll, _i, _i]),
    "po_matmul": (_i, [_vp, _ll, _ll, _i, _vp, _ll, _ll, _i, _vp, _ll, _ll, _i, _i, _ll, _ll, _ll, _ll, _f, _f,
                       _vp, _sz, _vp]),
}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    """A pytorch_opt_b200 C-ABI call failed."""


def load() -> ctypes.CDLL:
    """Load the shared library (raises if it is missing or incomplete)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeError(f"{LIB_PATH} is missing; build it with `python -m pytorch_opt_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                raise NativeError(f"{LIB_PATH} does not export {name}")
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().po_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != 0:
        raise NativeError(f"{what} failed (status {status}): {last_error()}")


def device_error(reset: bool = True) -> int:
    """Synchronise the current device and return (and clear) the device error word."""
    return int(load().po_device_error(1 if reset else 0))


GEMM_PROFILE_SLOTS = ("mma_full_wait", "mma_tempty_wait", "mma_total", "producer_empty_wait", "producer_total",
                      "epilogue_full_wait", "epilogue_work", "epilogue_total", "tiles")


def gemm_profile(enable: bool, read: bool = True) -> dict | None:
    """Switch the two-SM GEMM kernel's wait counters on or off; with `read`,
    first return (and zero) what they have summed (SM clock cycles)."""
    if not read:
        check(load().po_gemm_profile(1 if enable else 0, None, 0), "po_gemm_profile")
        return None
    out = (ctypes.c_ulonglong * 16)()
    check(load().po_gemm_profile(1 if enable else 0, ctypes.cast(out, ctypes.c_void_p), 16), "po_gemm_profile")
    return {name: int(out[i]) for i, name in enumerate(GEMM_PROFILE_SLOTS)}


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
