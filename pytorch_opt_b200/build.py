"""Build the sm_100a shared library ``libpytorch_opt_b200.so`` in-tree with nvcc.

The library is plain C ABI (``include/pytorch_opt_b200.h``); no torch headers
are involved, so it builds without a GPU and without torch's extension
machinery. Object files go to ``_build/`` at the repository root; the linked
library lands next to this file so that it ships with the package.

Usage: ``python -m pytorch_opt_b200.build [--force] [--debug]``
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(REPO_DIR, "_build")
LIB_NAME = "libpytorch_opt_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                "-I", INCLUDE, "-I", CSRC]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build pytorch_opt_b200")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return sorted(hs)


def _fingerprint(flags: list[str]) -> str:
    h = hashlib.sha256()
    for p in _sources() + _headers():
        with open(p, "rb") as f:
            h.update(p.encode())
            h.update(f.read())
    h.update(" ".join(flags).encode())
    return h.hexdigest()


# Sources compiled into the Newton-Schulz / Muon step (the benchmark's
# kernels): the product kernels, their launchers, the NS and Muon drivers and
# the elementwise passes.
NS_PATH_SOURCES = ("gemm.cuh", "gemm_pair.cuh", "gemm.cu", "gemm_launch.cuh", "gemm_pair_launch.cuh",
                   "gemm_host.cuh", "gemm_inst_", "ptx.cuh", "common.cuh", "ns.cu", "muon.cu", "elementwise.cu",
                   "elementwise.cuh")


def source_fingerprint(debug: bool = False, only=None) -> str:
    """Short hash of the library's sources, headers and compiler flags (what a
    build of the current tree contains); with ``only`` (file-name prefixes),
    of those csrc files alone. Profile summaries record the fingerprint of the
    kernels they profiled, so a figure taken from them can be matched to the
    build it describes."""
    flags = ARCH_FLAGS + COMMON_FLAGS + (["-DPO_DEBUG=1"] if debug else [])
    h = hashlib.sha256()
    files = _sources() + _headers()
    if only is not None:
        files = [p for p in files if os.path.dirname(p) == CSRC and os.path.basename(p).startswith(tuple(only))]
    for p in files:
        with open(p, "rb") as f:
            h.update(os.path.relpath(p, REPO_DIR).encode())
            h.update(f.read())
    h.update(" ".join(f for f in flags if not f.startswith(REPO_DIR)).encode())
    return h.hexdigest()[:16]


def build(force: bool = False, debug: bool = False, verbose: bool = False, jobs: int | None = None) -> str:
    """Compile every ``csrc/*.cu`` for sm_100a and link the shared library.

    Returns the library path. Skips the build when the sources, headers and
    flags are unchanged since the last successful build.
    """
    flags = ARCH_FLAGS + COMMON_FLAGS + (["-DPO_DEBUG=1"] if debug else [])
    stamp = LIB_PATH + ".stamp"
    fp = _fingerprint(flags)
    if not force and os.path.exists(LIB_PATH) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == fp:
                return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = _sources()
    objs = [os.path.join(BUILD_DIR, os.path.basename(s)[:-3] + ".o") for s in srcs]

    hdr_hash = hashlib.sha256()
    for p in _headers():
        with open(p, "rb") as f:
            hdr_hash.update(p.encode())
            hdr_hash.update(f.read())
    hdr_hash.update(" ".join(flags).encode())

    def obj_fingerprint(src: str) -> str:
        h = hdr_hash.copy()
        with open(src, "rb") as f:
            h.update(f.read())
        return h.hexdigest()

    def compile_one(pair):
        src, obj = pair
        ofp = obj_fingerprint(src)
        ostamp = obj + ".stamp"
        if not force and os.path.exists(obj) and os.path.exists(ostamp):
            with open(ostamp) as f:
                if f.read().strip() == ofp:
                    return obj  # unchanged since its last compile
        cmd = [nvcc, *flags, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
        with open(ostamp, "w") as f:
            f.write(ofp)
        return obj

    workers = jobs or min(len(srcs), os.cpu_count() or 4)
    # The tensor-core GEMM instantiations take longest: start them first.
    order = sorted(zip(srcs, objs), key=lambda so: (not os.path.basename(so[0]).startswith("gemm_inst"), so[0]))
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        list(ex.map(compile_one, order))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    with open(stamp, "w") as f:
        f.write(fp)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, debug=args.debug, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
