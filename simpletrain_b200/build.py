"""Build the sm_100a KDA library in-tree: ``simpletrain_b200/_lib/libkda_sm100.so``
(plain nvcc, one shared object exporting the C ABI of ``include/kda_sm100.h``)
and the torch ops over it, ``simpletrain_b200/_lib/kda_b200_ops.so``.

    python -m simpletrain_b200.build            # build if sources changed
    python -m simpletrain_b200.build --force    # rebuild

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


TORCH_OPS = os.path.join(LIBDIR, "kda_b200_ops.so")
TORCH_OPS_SRC = os.path.join(CSRC, "torch_ops.cpp")


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Build the torch dispatcher ops (``csrc/torch_ops.cpp``) against the C ABI
    library into ``_lib/kda_b200_ops.so`` (in-tree, loaded by ``simpletrain_b200.ops``)."""
    import torch

    h = hashlib.sha256()
    for f in (TORCH_OPS_SRC, os.path.join(ROOT, "include", "kda_sm100.h"), os.path.join(ROOT, "include", "st_fused_ops.h")):
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(torch.__version__.encode())
    digest = h.hexdigest()
    stamp = TORCH_OPS + ".srchash"
    if not force and os.path.exists(TORCH_OPS) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == digest:
                return TORCH_OPS
    bdir = os.path.join(LIBDIR, "_torch_build")
    os.makedirs(bdir, exist_ok=True)
    # compile in a child process: torch's loader registers the ops in the
    # process that builds them, and they may be registered only once per process
    code = (
        "from torch.utils.cpp_extension import load\n"
        f"load(name='kda_b200_ops', sources=[{TORCH_OPS_SRC!r}], build_directory={bdir!r}, with_cuda=True,\n"
        f"     extra_cflags=['-O2'], extra_include_paths=[{os.path.join(ROOT, 'include')!r}],\n"
        # $ORIGIN escaped for ninja ($$) and the shell (\\): the C ABI library sits beside this one
        f"     extra_ldflags=['-L{LIBDIR}', '-lkda_sm100', '-Wl,-rpath,\\\\$$ORIGIN:\\\\$$ORIGIN/..'],\n"
        f"     is_python_module=False, verbose={bool(verbose)})\n")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("torch ops build failed:\n" + res.stdout + res.stderr)
    shutil.copyfile(os.path.join(bdir, "kda_b200_ops.so"), TORCH_OPS + ".tmp")
    os.replace(TORCH_OPS + ".tmp", TORCH_OPS)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return TORCH_OPS


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
    if not args.trace:
        print(build_torch_ops(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    sys.exit(main())
