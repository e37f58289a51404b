"""Build the sm_100a KDA library in-tree: ``simpletrain_b200/_lib/libkda_sm100.so``.

    python -m simpletrain_b200.build            # build if sources changed
    python -m simpletrain_b200.build --force    # rebuild

Plain nvcc, one shared object exporting the C ABI of ``include/kda_sm100.h``.
Cross-compiles without a GPU.
"""
from __future__ import annotations

import argparse
import glob
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libkda_sm100.so")
STAMP = LIB + ".srchash"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O2",
              "--expt-relaxed-constexpr", "-Xptxas", "-O3"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _hash() -> str:
    h = hashlib.sha256()
    files = sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")))
    files.append(os.path.join(ROOT, "include", "kda_sm100.h"))
    for f in files:
        h.update(f.encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()


TRACE_LIB = os.path.join(LIBDIR, "libkda_sm100_trace.so")


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    """Build the library; ``trace=True`` builds the development variant with
    pipeline-event tracing into ``_lib/libkda_sm100_trace.so`` instead."""
    os.makedirs(LIBDIR, exist_ok=True)
    lib, stamp = (TRACE_LIB, TRACE_LIB + ".srchash") if trace else (LIB, STAMP)
    digest = _hash()
    if not force and os.path.exists(lib) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == digest:
                return lib
    tmp = lib + ".tmp"
    extra = ["-DKDA_TRACE"] if trace else []
    cmd = [nvcc_path(), *ARCH, *NVCC_FLAGS, *extra, "-I", os.path.join(ROOT, "include"), "-o", tmp, *sources()]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    os.replace(tmp, lib)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return lib


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build the tracing development variant")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose, trace=args.trace))


if __name__ == "__main__":
    sys.exit(main())
