"""TEST INFRASTRUCTURE ONLY — compile the reference's own native ATen source.

Builds kavinravi/pytorch-opt's ``pytorch_opt/ops/csrc/pytorch_opt_ops.cpp``
(its C++/ATen ops, bound with pybind11) with g++ directly from where it lies
in the reference checkout, into ``oracle/_ref/`` (git-ignored; the built
module travels with the tree to machines without the reference). Nothing is
copied from the reference into this repository. The module is the
"reference" CPU baseline of ``bench.py`` and a cross-check of the oracle.

    PYTORCH_OPT_REF=/path/to/pytorch-opt python oracle/build_ref.py
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MODULE = "pytorch_opt_native"
REL_SRC = os.path.join("pytorch_opt", "ops", "csrc", "pytorch_opt_ops.cpp")


def target_path() -> str:
    return os.path.join(OUT_DIR, MODULE + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build(ref_root: str | None = None, force: bool = False, verbose: bool = False) -> str | None:
    """Compile the reference extension; returns its path, or None when the source is absent."""
    ref_root = ref_root or os.environ.get("PYTORCH_OPT_REF")
    if not ref_root:
        return target_path() if os.path.exists(target_path()) else None
    src = os.path.join(ref_root, REL_SRC)
    if not os.path.exists(src):
        return target_path() if os.path.exists(target_path()) else None
    out = target_path()
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
        return out
    import torch
    from torch.utils import cpp_extension

    os.makedirs(OUT_DIR, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-shared", "-fPIC", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for inc in cpp_extension.include_paths():
        cmd += ["-isystem", inc]
    cmd += ["-isystem", sysconfig.get_paths()["include"], src, "-o", out + ".tmp"]
    for lib in cpp_extension.library_paths():
        cmd += ["-L", lib, f"-Wl,-rpath,{lib}"]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, capture_output=not verbose)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    path = build(sys.argv[1] if len(sys.argv) > 1 else None, force="--force" in sys.argv, verbose=True)
    print(path or "reference source not found (set PYTORCH_OPT_REF)")
