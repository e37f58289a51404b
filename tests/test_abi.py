"""The C ABI library: loads, exports what include/kda_sm100.h declares, and
the ctypes mirror has the C layout.  No kernel launches (runs without a GPU)."""
import ctypes
import os
import re
import shutil
import subprocess
import sys
import tempfile

import pytest

from simpletrain_b200 import _ffi

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADER = os.path.join(ROOT, "include", "kda_sm100.h")
HEADERS = (HEADER, os.path.join(ROOT, "include", "st_fused_ops.h"))


def _declared_functions():
    names = []
    for h in HEADERS:
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*((?:kda|st)_[a-z0-9_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _ffi.load()
    declared = _declared_functions()
    assert set(declared) >= set(_ffi.EXPORTED), declared
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert lib.kda_abi_version() == _ffi.ABI_VERSION


def test_nm_shows_c_linkage():
    if shutil.which("nm") is None:
        pytest.skip("nm not available")
    out = subprocess.run(["nm", "-D", "--defined-only", _ffi.LIB_PATH], capture_output=True, text=True).stdout
    for name in _declared_functions():
        assert re.search(rf"\bT {name}$", out, flags=re.M), name


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_ctypes_structs_match_c_layout():
    probe = r"""
#include <stdio.h>
#include <stddef.h>
#include "kda_sm100.h"
#define F(s, m) printf(#s "." #m " %zu\n", offsetof(s, m));
int main(void) {
  printf("kda_tensor %zu\nkda_fwd_params %zu\nkda_bwd_params %zu\n",
         sizeof(kda_tensor), sizeof(kda_fwd_params), sizeof(kda_bwd_params));
  F(kda_fwd_params, q) F(kda_fwd_params, y) F(kda_fwd_params, decay) F(kda_fwd_params, decay_scalar)
  F(kda_fwd_params, state_in) F(kda_fwd_params, workspace_bytes) F(kda_fwd_params, status)
  F(kda_bwd_params, q) F(kda_bwd_params, dg) F(kda_bwd_params, decay) F(kda_bwd_params, decay_scalar)
  F(kda_bwd_params, state_in) F(kda_bwd_params, dstate_out) F(kda_bwd_params, ddecay) F(kda_bwd_params, status)
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(probe)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.rsplit(" ", 1) for l in lines if l)
    assert int(got["kda_tensor"]) == ctypes.sizeof(_ffi.KdaTensor)
    assert int(got["kda_fwd_params"]) == ctypes.sizeof(_ffi.KdaFwdParams)
    assert int(got["kda_bwd_params"]) == ctypes.sizeof(_ffi.KdaBwdParams)
    for key, val in got.items():
        if "." in key:
            sname, field = key.split(".")
            cls = {"kda_fwd_params": _ffi.KdaFwdParams, "kda_bwd_params": _ffi.KdaBwdParams}[sname]
            assert getattr(cls, field).offset == int(val), key


def _fwd_params(**kw):
    p = _ffi.KdaFwdParams()
    p.B, p.H, p.T, p.D, p.chunk, p.dtype = 1, 1, 64, 64, 64, _ffi.KDA_DTYPE_BF16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    (dict(D=96), _ffi.KDA_ERR_UNSUPPORTED),
    (dict(chunk=32), _ffi.KDA_ERR_UNSUPPORTED),
    (dict(dtype=7), _ffi.KDA_ERR_UNSUPPORTED),
    (dict(flags=1 << 5), _ffi.KDA_ERR_UNSUPPORTED),
    (dict(T=-1), _ffi.KDA_ERR_BAD_SHAPE),
    (dict(D=128, flags=_ffi.KDA_FLAG_LITERAL), _ffi.KDA_ERR_BAD_SHAPE),
    (dict(B=0), _ffi.KDA_OK),       # empty batch: nothing to do, no pointers touched
    (dict(H=0), _ffi.KDA_OK),
])
def test_forward_argument_checks(kw, code):
    lib = _ffi.load()
    assert lib.kda_fwd_sm100(ctypes.byref(_fwd_params(**kw)), None) == code


@pytest.mark.parametrize("kw,code", [
    (dict(D=96), _ffi.KDA_ERR_UNSUPPORTED),
    (dict(chunk=32), _ffi.KDA_ERR_UNSUPPORTED),
    (dict(T=-1), _ffi.KDA_ERR_BAD_SHAPE),
    (dict(D=128, flags=_ffi.KDA_FLAG_LITERAL), _ffi.KDA_ERR_BAD_SHAPE),
    (dict(), _ffi.KDA_ERR_NULL_ARGUMENT),
    (dict(B=0), _ffi.KDA_OK),       # nothing to do: no scratch looked up, no pointers touched
])
def test_noalloc_checks_arguments_like_the_forward(kw, code):
    lib = _ffi.load()
    assert lib.kda_fwd_sm100_noalloc(ctypes.byref(_fwd_params(**kw)), None) == code
    assert lib.kda_fwd_sm100(ctypes.byref(_fwd_params(**kw)), None) == code
    assert lib.kda_fwd_sm100_noalloc(None, None) == _ffi.KDA_ERR_NULL_ARGUMENT


_NOALLOC_ORDER_CHILD = r"""
import ctypes
from simpletrain_b200 import _ffi
lib = _ffi.load()
good = _ffi.KdaTensor(0x10000, 64 * 128, 64 * 128, 128, 1)
p = _ffi.KdaFwdParams()
p.B, p.H, p.T, p.D, p.chunk, p.dtype = 1, 600, 64, 128, 64, _ffi.KDA_DTYPE_BF16
p.q = p.k = p.v = p.y = good
need = lib.kda_fwd_workspace_bytes(1, 600, 64, 128, 64, 0)
rc_big = lib.kda_fwd_sm100_noalloc(ctypes.byref(p), None)
p.q = _ffi.KdaTensor(0x10008, 64 * 128, 64 * 128, 128, 1)      # misaligned, and still too big
rc_bad = lib.kda_fwd_sm100_noalloc(ctypes.byref(p), None)
print(need, rc_big, rc_bad, lib.kda_launch_count())
"""


def test_noalloc_reports_bad_arguments_before_its_size_limit():
    """A problem over the scratch limit (forced with one work range per chunk)
    is refused with KDA_ERR_WORKSPACE, but an argument error wins over it; nothing
    is launched (the pointers are never touched)."""
    env = dict(os.environ, KDA_SM100_RANGES="600")
    out = subprocess.run([sys.executable, "-c", _NOALLOC_ORDER_CHILD], env=env, cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    need, rc_big, rc_bad, launched = (int(x) for x in out.stdout.split())
    assert need > _ffi.NOALLOC_SCRATCH_BYTES
    assert rc_big == _ffi.KDA_ERR_WORKSPACE
    assert rc_bad == _ffi.KDA_ERR_BAD_LAYOUT
    assert launched == 0


def _bwd_params(**kw):
    p = _ffi.KdaBwdParams()
    p.B, p.H, p.T, p.D, p.chunk, p.dtype = 1, 1, 64, 64, 64, _ffi.KDA_DTYPE_BF16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw", [
    dict(flags=_ffi.KDA_FLAG_PER_STEP | _ffi.KDA_FLAG_LITERAL),            # two semantics at once
    dict(flags=_ffi.KDA_FLAG_PER_STEP, decay_scalar=0.1),                   # below the row-scaling range
    dict(flags=_ffi.KDA_FLAG_PER_STEP, decay_scalar=1.5),
    dict(flags=_ffi.KDA_FLAG_PER_STEP, decay_scalar=0.8, dtype=_ffi.KDA_DTYPE_F16),   # fp16 range
    dict(flags=_ffi.KDA_FLAG_PER_STEP, decay=0x10000, decay_stride_d=1),    # varies along the key channels
])
def test_per_step_argument_checks(kw):
    lib = _ffi.load()
    assert lib.kda_fwd_sm100(ctypes.byref(_fwd_params(**kw)), None) == _ffi.KDA_ERR_UNSUPPORTED
    assert lib.kda_bwd_sm100(ctypes.byref(_bwd_params(**kw)), None) == _ffi.KDA_ERR_UNSUPPORTED


def test_per_step_backward_has_no_decay_gradient():
    lib = _ffi.load()
    p = _bwd_params(flags=_ffi.KDA_FLAG_PER_STEP, decay_scalar=0.9, ddecay=0x10000)
    assert lib.kda_bwd_sm100(ctypes.byref(p), None) == _ffi.KDA_ERR_UNSUPPORTED


def test_null_params_and_missing_tensors():
    lib = _ffi.load()
    assert lib.kda_fwd_sm100(None, None) == _ffi.KDA_ERR_NULL_ARGUMENT
    assert lib.kda_bwd_sm100(None, None) == _ffi.KDA_ERR_NULL_ARGUMENT
    # q is NULL while there is work to do
    assert lib.kda_fwd_sm100(ctypes.byref(_fwd_params()), None) == _ffi.KDA_ERR_NULL_ARGUMENT


def test_layout_rules_are_enforced_before_any_launch():
    lib = _ffi.load()
    good = _ffi.KdaTensor(0x10000, 64 * 64, 64 * 64, 64, 1)
    p = _fwd_params(q=good, k=good, v=good, y=good)
    p.q = _ffi.KdaTensor(0x10000, 64 * 64, 64 * 64, 64, 2)      # strided innermost dim
    assert lib.kda_fwd_sm100(ctypes.byref(p), None) == _ffi.KDA_ERR_BAD_LAYOUT
    p.q = _ffi.KdaTensor(0x10008, 64 * 64, 64 * 64, 64, 1)      # 8-byte aligned base
    assert lib.kda_fwd_sm100(ctypes.byref(p), None) == _ffi.KDA_ERR_BAD_LAYOUT
    p.q = _ffi.KdaTensor(0x10000, 64 * 64, 64 * 64, 65, 1)      # token stride not 16-byte multiple
    assert lib.kda_fwd_sm100(ctypes.byref(p), None) == _ffi.KDA_ERR_BAD_LAYOUT


def test_workspace_sizes_and_status_strings():
    lib = _ffi.load()
    # one fp32 state handoff slot per boundary between work ranges; 6 streams of 2
    # chunks here: cut ranges hold at least 4 chunks, so one range per stream, 7 boundaries
    assert lib.kda_fwd_workspace_bytes(2, 3, 128, 128, 64, 0) >= 7 * 128 * 128 * 4
    assert lib.kda_bwd_workspace_bytes(2, 3, 128, 128, 64, 0) >= 7 * 3 * 128 * 128 * 4
    # one stream of 256 chunks: 64 ranges of 4 chunks (not one per CTA slot), each with
    # a boundary slot and a range aggregate of 64 KiB
    slot = 128 * 128 * 4
    assert 129 * slot <= lib.kda_fwd_workspace_bytes(1, 1, 256 * 64, 128, 64, 0) < 130 * slot
    # bounded by the CTA count, not by the problem size
    assert lib.kda_fwd_workspace_bytes(64, 64, 1 << 16, 128, 64, 0) < 64 << 20
    assert lib.kda_fwd_workspace_bytes(0, 3, 128, 128, 64, 0) < 1024
    for code in (0, 1, 2, 3, 4, 5, 6, 64):
        s = _ffi.status_string(code)
        assert s and s != "unknown kda status"
    assert _ffi.status_string(12345) == "unknown kda status"
