"""ctypes binding of ``include/kda_sm100.h`` (the library's C ABI).

The structures below mirror the header field for field; ``ABI_VERSION`` must
match ``KDA_ABI_VERSION``.  Loading fails loudly when the library has not been
built -- there is no other implementation to fall back to.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_int32, c_int64, c_size_t, c_uint32, c_void_p

ABI_VERSION = 2
# KDA_B200_LIB_DIR selects another build of both libraries (default: in-tree _lib/)
LIB_DIR = os.environ.get("KDA_B200_LIB_DIR") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libkda_sm100.so")

KDA_DTYPE_BF16 = 0
KDA_DTYPE_F16 = 1
KDA_FLAG_LITERAL = 1 << 0
KDA_FLAG_PER_STEP = 1 << 1

KDA_OK = 0
KDA_ERR_NULL_ARGUMENT = 1
KDA_ERR_BAD_SHAPE = 2
KDA_ERR_UNSUPPORTED = 3
KDA_ERR_BAD_LAYOUT = 4
KDA_ERR_WORKSPACE = 5
KDA_ERR_CUDA = 6
KDA_ERR_DEVICE_TIMEOUT = 64

EXPORTED = (
    "kda_fwd_sm100", "kda_bwd_sm100", "kda_fwd_workspace_bytes", "kda_bwd_workspace_bytes",
    "kda_status_string", "kda_abi_version", "kda_launch_count", "kda_fwd_sm100_noalloc",
    "kda_trace_start", "kda_trace_read", "kda_trace_stop", "kda_kernel_name",
    # include/st_fused_ops.h
    "st_silu_mul_fwd", "st_silu_mul_bwd", "st_rmsnorm_residual_fwd", "st_rmsnorm_residual_bwd",
    "st_rmsnorm_residual_bwd_scratch", "st_cross_entropy_fwd", "st_cross_entropy_bwd",
)
NOALLOC_SCRATCH_BYTES = 32 << 20


class KdaTensor(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("stride_b", c_int64), ("stride_h", c_int64),
                ("stride_t", c_int64), ("stride_d", c_int64)]


class KdaFwdParams(ctypes.Structure):
    _fields_ = [
        ("B", c_int32), ("H", c_int32), ("T", c_int32), ("D", c_int32),
        ("chunk", c_int32), ("dtype", c_int32), ("flags", c_uint32),
        ("q", KdaTensor), ("k", KdaTensor), ("v", KdaTensor), ("g", KdaTensor), ("y", KdaTensor),
        ("decay", c_void_p), ("decay_stride_b", c_int64), ("decay_stride_h", c_int64),
        ("decay_stride_d", c_int64), ("decay_scalar", c_double),
        ("state_in", c_void_p), ("state_out", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("status", c_void_p),
    ]


class KdaBwdParams(ctypes.Structure):
    _fields_ = [
        ("B", c_int32), ("H", c_int32), ("T", c_int32), ("D", c_int32),
        ("chunk", c_int32), ("dtype", c_int32), ("flags", c_uint32),
        ("q", KdaTensor), ("k", KdaTensor), ("v", KdaTensor), ("g", KdaTensor), ("dy", KdaTensor),
        ("dq", KdaTensor), ("dk", KdaTensor), ("dv", KdaTensor), ("dg", KdaTensor),
        ("decay", c_void_p), ("decay_stride_b", c_int64), ("decay_stride_h", c_int64),
        ("decay_stride_d", c_int64), ("decay_scalar", c_double),
        ("state_in", c_void_p), ("dstate_out", c_void_p),
        ("dstate_in", c_void_p), ("ddecay", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("status", c_void_p),
    ]


_LIB = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the KDA library (once) and declare its signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(
            f"KDA sm_100a library not found at {path}; build it with "
            "`python -m simpletrain_b200.build` (needs nvcc)")
    lib = ctypes.CDLL(path)
    lib.kda_fwd_sm100.argtypes = [POINTER(KdaFwdParams), c_void_p]
    lib.kda_fwd_sm100.restype = c_int32
    lib.kda_bwd_sm100.argtypes = [POINTER(KdaBwdParams), c_void_p]
    lib.kda_bwd_sm100.restype = c_int32
    for fn in (lib.kda_fwd_workspace_bytes, lib.kda_bwd_workspace_bytes):
        fn.argtypes = [c_int32, c_int32, c_int32, c_int32, c_int32, c_uint32]
        fn.restype = c_size_t
    lib.kda_status_string.argtypes = [c_int32]
    lib.kda_status_string.restype = c_char_p
    lib.kda_abi_version.argtypes = []
    lib.kda_abi_version.restype = c_int32
    lib.kda_launch_count.argtypes = []
    lib.kda_launch_count.restype = ctypes.c_uint64
    lib.kda_fwd_sm100_noalloc.argtypes = [POINTER(KdaFwdParams), c_void_p]
    lib.kda_fwd_sm100_noalloc.restype = c_int32
    lib.kda_trace_start.argtypes = [c_int32]
    lib.kda_trace_start.restype = c_int32
    for fn in (lib.kda_trace_read, lib.kda_trace_stop):
        fn.argtypes = [POINTER(ctypes.c_float), POINTER(c_int32), c_int32]
        fn.restype = c_int32
    lib.kda_kernel_name.argtypes = [c_int32]
    lib.kda_kernel_name.restype = c_char_p
    ver = lib.kda_abi_version()
    if ver != ABI_VERSION:
        raise ImportError(f"KDA library ABI version {ver} != binding version {ABI_VERSION}; rebuild")
    _LIB = lib
    return lib


def status_string(code: int) -> str:
    return load().kda_status_string(int(code)).decode()


def launch_count() -> int:
    """Kernels the library has launched in this process."""
    return int(load().kda_launch_count())


class KernelTrace:
    """CUDA-event device time of each KDA kernel launched inside the block.

        with KernelTrace(max_launches=4096) as tr:
            ...                                 # calls into the library
        tr.launches                             # [(kernel name, ms), ...] in launch order
        tr.per_kernel()                         # {name: (launches, mean ms)}

    The events are recorded on each kernel's launching stream by the library
    itself (``kda_trace_start`` / ``kda_trace_stop``), so every kernel of a
    multi-kernel call (the backward's two passes) is timed on its own.

    Launches captured into a CUDA graph inside the block are timed at every
    replay: call ``read()`` after each replay has finished (it appends that
    replay's launches), and destroy the graph before the block ends.
    """

    def __init__(self, max_launches: int = 4096):
        self.max = int(max_launches)
        self.launches = []
        self._read = False

    def _collect(self, fn):
        lib = load()
        ms = (ctypes.c_float * self.max)()
        ids = (c_int32 * self.max)()
        n = fn(ms, ids, self.max)
        if n < 0:
            raise RuntimeError(f"kernel trace: {status_string(-n)}")
        n = min(n, self.max)
        return [(lib.kda_kernel_name(ids[i]).decode(), float(ms[i])) for i in range(n) if ids[i] >= 0]

    def read(self):
        """Append the launches recorded so far (a graph's: those of its last replay)."""
        self._read = True
        got = self._collect(load().kda_trace_read)
        self.launches += got
        return got

    def __enter__(self):
        rc = load().kda_trace_start(self.max)
        if rc != KDA_OK:
            raise RuntimeError(f"kda_trace_start: {status_string(rc)}")
        return self

    def __exit__(self, *exc):
        got = self._collect(load().kda_trace_stop)
        if not self._read:
            self.launches = got
        return False

    def per_kernel(self):
        out = {}
        for name, t in self.launches:
            c, s = out.get(name, (0, 0.0))
            out[name] = (c + 1, s + t)
        return {n: (c, s / c) for n, (c, s) in out.items()}
