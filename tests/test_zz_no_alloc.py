"""kda_fwd_sm100_noalloc: the forward scan for callers that cannot allocate.

Some callers of this C ABI cannot allocate device memory for a workspace (a
host runtime that only holds the tensors it was given, or a process whose
device memory is reserved up front).  The no-allocation entry point takes the
same parameters as kda_fwd_sm100 and draws its scratch from a fixed device
array inside the library.  These tests call it through the C ABI and check it
against the allocating entry point on two calls in a row (the array keeps the
previous call's contents, so the second call checks that each call resets
what it must), and that oversized problems are refused before any launch.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

from oracle.kda_oracle import max_rel
from simpletrain_b200 import _ffi, device_status
from simpletrain_b200.ops import _DTYPES, _decay_fields, _desc, _ptr, status_word
from simpletrain_b200.workloads import custom, make_inputs

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

TOL_LOWP = 2e-2    # bf16 outputs, normwise max|x-ref|/max|ref|
TOL_STATE = 1e-3   # fp32 final state


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _params(q, k, v, g, decay_bhd, s0, y, s_out, literal=False):
    B, H, T, D = q.shape
    dptr, dsb, dsh, dsd = _decay_fields(decay_bhd)
    return _ffi.KdaFwdParams(
        B, H, T, D, 64, _DTYPES[q.dtype], _ffi.KDA_FLAG_LITERAL if literal else 0,
        _desc(q), _desc(k), _desc(v), _desc(g), _desc(y),
        dptr, dsb, dsh, dsd, 0.0,
        _ptr(s0), _ptr(s_out), None, 0, status_word(q.device).data_ptr())


def _noalloc(q, k, v, g, decay_bhd, s0):
    B, H, T, D = q.shape
    y = torch.empty_like(q)
    s_out = torch.empty(B, H, D, D, dtype=torch.float32, device=q.device)
    p = _params(q, k, v, g, decay_bhd, s0, y, s_out)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _ffi.load().kda_fwd_sm100_noalloc(ctypes.byref(p), stream)
    assert rc == _ffi.KDA_OK, _ffi.status_string(rc)
    return y, s_out


@pytest.mark.parametrize("B,H,T,D", [
    (4, 6, 600, 128), (16, 10, 512, 128), (3, 5, 1000, 64),
    (1, 2, 4096, 128),   # long streams: range aggregates and folded entries in the scratch too
])
def test_noalloc_matches_allocating_entry_point_twice(B, H, T, D):
    w = custom(B, H, T, D, backward=False, s0_std=0.02)
    inp = make_inputs(w, seed=3, device="cuda")
    q, k, v, g, s0 = inp["q"], inp["k"], inp["v"], inp["g"], inp["s0"]
    dec = inp["decay"].expand(B, H, D)
    y_ref, s_ref = torch.ops.kda_b200.chunk_fwd(q, k, v, g, dec, 0.0, s0, 64, 0, True)
    for _ in range(2):
        y, s = _noalloc(q, k, v, g, dec, s0)
        torch.cuda.synchronize()
        assert device_status() == 0
        assert max_rel(y.float().cpu(), y_ref.float().cpu()) <= TOL_LOWP
        assert max_rel(s.cpu(), s_ref.cpu()) <= TOL_STATE


def test_default_schedules_fit_the_scratch():
    """The scratch a forward needs is bounded by the device's CTA slots, not by
    the problem: with the default schedule every shape fits the fixed array --
    many short streams (one range per CTA slot, the D=64 kernels run two CTAs
    per SM), a few long streams (range aggregates), each semantics."""
    lib = _ffi.load()
    shapes = [(64, 64, 64), (16, 10, 2048), (16, 8, 2048), (1, 1, 1 << 20), (1, 28, 32768), (3, 1, 64 * 1000)]
    for D in (64, 128):
        flag_sets = [0, _ffi.KDA_FLAG_PER_STEP] + ([_ffi.KDA_FLAG_LITERAL] if D == 64 else [])
        for flags in flag_sets:
            for B, H, T in shapes:
                need = lib.kda_fwd_workspace_bytes(B, H, T, D, 64, flags)
                assert need <= _ffi.NOALLOC_SCRATCH_BYTES, (B, H, T, D, flags, need)


_OVERSIZE_CHILD = r"""
import ctypes
from simpletrain_b200 import _ffi
lib = _ffi.load()
B, H, T, D = 1, 600, 64, 128          # 600 single-chunk streams, one range each
need = lib.kda_fwd_workspace_bytes(B, H, T, D, 64, 0)
p = _ffi.KdaFwdParams()
p.B, p.H, p.T, p.D, p.chunk, p.dtype = B, H, T, D, 64, _ffi.KDA_DTYPE_BF16
# well-formed views (never dereferenced: the size check refuses the call first)
p.q = p.k = p.v = p.y = _ffi.KdaTensor(0x10000, T * D * H, T * D, D, 1)
before = _ffi.launch_count()
rc = lib.kda_fwd_sm100_noalloc(ctypes.byref(p), None)
print(need, rc, _ffi.launch_count() - before)
"""


def test_noalloc_rejects_problems_larger_than_its_scratch():
    # The scratch holds one state slot per boundary between work ranges, and by
    # default there is one range per resident CTA, which stays far below the
    # limit; KDA_SM100_RANGES forces one range per chunk in a child process.
    env = dict(os.environ, KDA_SM100_RANGES="600")
    out = subprocess.run([sys.executable, "-c", _OVERSIZE_CHILD], env=env, cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    need, rc, launched = (int(x) for x in out.stdout.split())
    assert need > _ffi.NOALLOC_SCRATCH_BYTES
    assert rc == _ffi.KDA_ERR_WORKSPACE
    assert launched == 0                       # refused before anything was enqueued
