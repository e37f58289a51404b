"""Parity of the sm_100a KDA kernels with the CPU oracle (and the reference's
own golden vectors).

Tolerances (from the build's target): bf16/fp16 outputs and gradients within
normwise max-rel 2e-2 of the fp32 oracle, fp32 final state within 1e-3,
where  max_rel(x, ref) = max|x - ref| / max|ref|.
"""
import os

import pytest
import torch

from oracle.kda_oracle import chunk_scan, decay_bhd1, max_rel
from simpletrain_b200 import device_status, kda_chunk, kda_chunked_scan
from simpletrain_b200.workloads import WORKLOADS, custom, make_inputs

pytestmark = pytest.mark.gpu

TOL_LOWP = 2e-2     # bf16 / fp16 outputs and gradients
TOL_STATE = 1e-3    # fp32 final state
DEV = "cuda"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert device_status() == 0, "a device-side bounded wait expired"


def oracle(q, k, v, g, decay, s0, dy=None, dsT=None, mode="corrected", chunk=64):
    """fp32 oracle forward (+ autograd backward when dy is given) on CPU."""
    leaves = [t.detach().cpu().float().requires_grad_(dy is not None) for t in (q, k, v)]
    gl = g.detach().cpu().float().requires_grad_(dy is not None) if g is not None else None
    if torch.is_tensor(decay):
        dl = decay.detach().cpu().float().requires_grad_(dy is not None)
        B, H, _, D = q.shape
        dec = decay_bhd1(dl, B, H, D) if dl.dim() <= 3 else dl
    else:
        dl, dec = None, decay
    sl = s0.detach().cpu().float().requires_grad_(dy is not None) if s0 is not None else None
    y, S = chunk_scan(*leaves, gl, dec, chunk, initial_state=sl, mode=mode)
    out = {"y": y.detach(), "S": S.detach()}
    if dy is not None:
        loss = (y * dy.detach().cpu().float()).sum()
        if dsT is not None:
            loss = loss + (S * dsT.detach().cpu().float()).sum()
        loss.backward()
        out.update(dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad)
        if gl is not None:
            out["dg"] = gl.grad
        if dl is not None:
            out["ddecay"] = dl.grad
        if sl is not None:
            out["ds0"] = sl.grad
    return out


def run_gpu(q, k, v, g, decay, s0, dy=None, dsT=None, literal=False, want_state=True):
    leaves = [t.detach().to(DEV).requires_grad_(dy is not None) for t in (q, k, v)]
    gl = g.detach().to(DEV).requires_grad_(dy is not None) if g is not None else None
    dl = decay.detach().to(DEV).requires_grad_(dy is not None) if torch.is_tensor(decay) else decay
    sl = s0.detach().to(DEV).requires_grad_(dy is not None) if s0 is not None else None
    y, S = kda_chunk(*leaves, gl, dl, sl, 64, reference_exact=literal, output_final_state=want_state)
    out = {"y": y.detach(), "S": S.detach() if S is not None else None}
    if dy is not None:
        loss = (y.float() * dy.to(DEV).float()).sum()
        if dsT is not None:
            loss = loss + (S * dsT.to(DEV)).sum()
        loss.backward()
        out.update(dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad)
        if gl is not None:
            out["dg"] = gl.grad
        if torch.is_tensor(dl):
            out["ddecay"] = dl.grad
        if sl is not None:
            out["ds0"] = sl.grad
    return out


def compare(got, ref, keys=None):
    errs = {}
    for key in keys or ref.keys():
        if key not in got or got[key] is None:
            continue
        tol = TOL_STATE if key == "S" else TOL_LOWP
        e = max_rel(got[key].float().cpu(), ref[key])
        errs[key] = e
        assert e <= tol, f"{key}: max_rel {e:.3e} > {tol:.0e}  (all: {errs})"
    return errs


def _rand(B, H, T, D, dtype=torch.bfloat16, seed=0, gate=True):
    g = torch.Generator().manual_seed(seed)
    def mk():
        return torch.randn(B, T, H, D, generator=g).to(dtype).transpose(1, 2)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).to(dtype).transpose(1, 2)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).to(dtype).transpose(1, 2)
    v = mk()
    gt = torch.sigmoid(torch.randn(B, T, H, D, generator=g)).to(dtype).transpose(1, 2) if gate else None
    dy = mk()
    decay = torch.sigmoid(torch.randn(H, D, generator=g) + 3.0)
    return q, k, v, gt, dy, decay


# --------------------------------------------------------------------------- #
# small shapes, every option
# --------------------------------------------------------------------------- #
SMALL = [
    # B, H, T, D, gate, decay kind, s0, literal
    (2, 3, 256, 64, True, "channel", False, False),
    (1, 2, 200, 128, True, "channel", True, False),
    (2, 2, 130, 64, False, "scalar", False, False),
    (1, 3, 64, 128, True, "head", True, False),
    (1, 1, 1, 64, True, "channel", True, False),
    (1, 2, 77, 128, False, "scalar", True, False),
    (2, 2, 192, 64, True, "scalar", False, True),
    (1, 2, 256, 64, True, "channel", True, True),
]


@pytest.mark.parametrize("B,H,T,D,gate,dkind,with_s0,literal", SMALL)
def test_forward_small(B, H, T, D, gate, dkind, with_s0, literal):
    q, k, v, g, _, dch = _rand(B, H, T, D, gate=gate)
    decay = {"channel": dch, "scalar": 0.97, "head": dch[:, 0].contiguous()}[dkind]
    s0 = torch.randn(B, H, D, D) * 0.05 if with_s0 else None
    ref = oracle(q, k, v, g, decay, s0, mode="literal" if literal else "corrected")
    got = run_gpu(q, k, v, g, decay, s0, literal=literal)
    compare(got, ref, ["y", "S"])


@pytest.mark.parametrize("B,H,T,D,gate,dkind,with_s0,literal", SMALL)
def test_backward_small(B, H, T, D, gate, dkind, with_s0, literal):
    q, k, v, g, dy, dch = _rand(B, H, T, D, gate=gate, seed=1)
    decay = {"channel": dch, "scalar": 0.97, "head": dch[:, 0].contiguous()}[dkind]
    s0 = torch.randn(B, H, D, D) * 0.05 if with_s0 else None
    dsT = torch.randn(B, H, D, D) * 0.1
    ref = oracle(q, k, v, g, decay, s0, dy, dsT, mode="literal" if literal else "corrected")
    got = run_gpu(q, k, v, g, decay, s0, dy, dsT, literal=literal)
    compare(got, ref)


# --------------------------------------------------------------------------- #
# few streams, each much longer than a work range: the carry crosses chains of
# middle ranges through precomputed range aggregates
# --------------------------------------------------------------------------- #
LONG = [
    # B, H, T, D, gate, decay kind, s0, literal
    (1, 1, 4096, 128, True, "channel", True, False),
    (1, 2, 3000, 64, True, "scalar", False, False),
    (1, 2, 2048, 64, True, "channel", True, True),
    (2, 1, 2500, 128, False, "head", True, False),
]


@pytest.mark.parametrize("B,H,T,D,gate,dkind,with_s0,literal", LONG)
def test_long_streams_forward_and_backward(B, H, T, D, gate, dkind, with_s0, literal):
    q, k, v, g, dy, dch = _rand(B, H, T, D, gate=gate, seed=5)
    decay = {"channel": dch, "scalar": 0.995, "head": dch[:, 0].contiguous()}[dkind]
    s0 = torch.randn(B, H, D, D) * 0.02 if with_s0 else None
    dsT = torch.randn(B, H, D, D) * 0.1
    mode = "literal" if literal else "corrected"
    ref = oracle(q, k, v, g, decay, s0, dy, dsT, mode=mode)
    got = run_gpu(q, k, v, g, decay, s0, dy, dsT, literal=literal)
    compare(got, ref)


def test_fp16_inputs():
    q, k, v, g, dy, dch = _rand(1, 2, 160, 128, dtype=torch.float16, seed=2)
    ref = oracle(q, k, v, g, dch, None, dy)
    got = run_gpu(q, k, v, g, dch, None, dy)
    assert got["y"].dtype == torch.float16
    compare(got, ref)


def test_contiguous_bhtd_inputs_and_side_stream():
    q, k, v, g, dy, dch = _rand(2, 2, 128, 64, seed=3)
    q, k, v, g = (t.contiguous() for t in (q, k, v, g))
    ref = oracle(q, k, v, g, dch, None)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        got = run_gpu(q, k, v, g, dch, None)
    s.synchronize()
    compare(got, ref, ["y", "S"])


def test_empty_sequence_returns_initial_state():
    q = torch.empty(1, 2, 0, 64, dtype=torch.bfloat16, device=DEV)
    s0 = torch.randn(1, 2, 64, 64, device=DEV)
    y, S = kda_chunk(q, q, q, None, 0.9, s0)
    assert y.shape == q.shape and torch.equal(S, s0)


# --------------------------------------------------------------------------- #
# the reference's own golden vectors through the drop-in dispatch
# --------------------------------------------------------------------------- #
def test_dropin_matches_reference_golden_bf16(golden_dir):
    f = torch.load(os.path.join(golden_dir, "lit_bf16.pt"), weights_only=False)
    q, k, v, g = (f[n].to(DEV).requires_grad_(True) for n in ("q", "k", "v", "g"))
    decay = f["decay"].to(DEV).requires_grad_(True)
    y = kda_chunked_scan(q, k, v, gate=g, decay=decay, chunk_size=f["chunk"])
    assert y.dtype == torch.bfloat16 and y.shape == f["y"].shape
    (y.float() * f["dy"].to(DEV).float()).sum().backward()
    for name, got in (("y", y), ("dq", q.grad), ("dk", k.grad), ("dv", v.grad), ("dg", g.grad),
                      ("ddecay", decay.grad)):
        e = max_rel(got.float().cpu(), f[name].float())
        assert e <= TOL_LOWP, (name, e)


def test_decay_gradient_vanishes_when_decay_only_scales_zero_state():
    """Two chunks from a zero state: decay multiplies only the zero initial state
    and the unused final update, so d(loss)/d(decay) is exactly 0 in the
    reference; the closed form returns rounding noise far below the terms."""
    q, k, v, g, dy, dch = _rand(1, 2, 128, 64, seed=5)
    dl = dch.to(DEV).requires_grad_(True)
    y, _ = kda_chunk(q.to(DEV), k.to(DEV), v.to(DEV), g.to(DEV), dl, None, 64,
                     reference_exact=True, output_final_state=False)
    (y.float() * dy.to(DEV).float()).sum().backward()
    assert dl.grad.abs().max().item() < 1e-3


def test_dropin_matches_reference_golden_f32_inputs_cast(golden_dir):
    f = torch.load(os.path.join(golden_dir, "lit_f32.pt"), weights_only=False)
    cast = lambda t: t.to(DEV, torch.bfloat16)
    y = kda_chunked_scan(cast(f["q"]), cast(f["k"]), cast(f["v"]), cast(f["g"]), f["decay"], f["chunk"])
    assert max_rel(y.float().cpu(), f["y"]) <= TOL_LOWP


def test_dropin_rejects_fp32_like_reference():
    q = torch.randn(1, 1, 64, 64, device=DEV)
    with pytest.raises(AssertionError):
        kda_chunked_scan(q, q, q)


def test_dropin_layer_call_pattern():
    """The call KimiDeltaAttention.forward makes (models/kimi_k3.py:99-118)."""
    for H, Dh in ((8, 64), (10, 128)):
        B, T = 2, 256
        x = torch.randn(B, T, H * Dh, device=DEV, dtype=torch.bfloat16)
        q, k, v, g = (x.view(B, T, H, Dh).transpose(1, 2) * s for s in (1.0, 0.5, 0.25, 1.5))
        y = kda_chunked_scan(q, k, v, gate=g, decay=0.97, chunk_size=64, use_triton=True)
        assert y.shape == (B, H, T, Dh) and y.dtype == torch.bfloat16
        mode = "literal" if Dh == 64 else "corrected"
        ref = oracle(q, k, v, g, 0.97, None, mode=mode)
        assert max_rel(y.float().cpu(), ref["y"]) <= TOL_LOWP


# --------------------------------------------------------------------------- #
# the seeded workload shapes
# --------------------------------------------------------------------------- #
def _bh_slice(inp, bs, hs):
    out = {}
    for n in ("q", "k", "v", "g", "dy"):
        t = inp[n]
        out[n] = t[bs][:, hs] if t is not None else None
    out["decay"] = inp["decay"][hs]
    out["s0"] = inp["s0"][bs][:, hs] if inp["s0"] is not None else None
    return out


def test_config_100m_forward():
    w = WORKLOADS["100m-fwd"]
    inp = make_inputs(w, seed=0)
    got = run_gpu(inp["q"], inp["k"], inp["v"], inp["g"], inp["decay"], inp["s0"])
    ref = oracle(inp["q"], inp["k"], inp["v"], inp["g"], inp["decay"], inp["s0"])
    compare(got, ref, ["y", "S"])


def test_config_1b_forward_backward():
    w = WORKLOADS["1b-fwdbwd"]
    inp = make_inputs(w, seed=0)
    args = (inp["q"], inp["k"], inp["v"], inp["g"], inp["decay"], inp["s0"], inp["dy"])
    compare(run_gpu(*args), oracle(*args))


@pytest.mark.parametrize("name,heads", [("7b-fwdbwd", [0, 13, 23]), ("10b-fwdbwd", [0, 27])])
def test_config_large_forward_backward_head_subset(name, heads):
    """Full-size GPU run; the oracle checks a few (batch, head) pairs (heads are independent)."""
    w = WORKLOADS[name]
    inp = make_inputs(w, seed=0)
    got = run_gpu(inp["q"], inp["k"], inp["v"], inp["g"], inp["decay"], inp["s0"], inp["dy"])
    sub = _bh_slice(inp, slice(0, 1), heads)
    ref = oracle(sub["q"], sub["k"], sub["v"], sub["g"], sub["decay"], sub["s0"], sub["dy"])
    gsub = {}
    for n, t in got.items():
        if t is None:
            continue
        if n == "ddecay":
            gsub[n] = t[heads]          # decay is [H, D]: its gradient sums over the batch
        else:
            gsub[n] = t[0:1][:, heads]
    keys = ["y", "S", "dq", "dk", "dv", "dg", "ds0"]
    compare(gsub, ref, keys)
    if w.B == 1:
        compare(gsub, ref, ["ddecay"])


def test_long_context_split_consistency():
    """Size-independent check at the long-context shape: scanning [0, T/2) and
    then [T/2, T) from the handed-over state equals one scan over [0, T)."""
    w = WORKLOADS["10b-fwdbwd"]
    inp = make_inputs(w, seed=0, device=DEV)
    q, k, v, g, decay, s0 = (inp[n] for n in ("q", "k", "v", "g", "decay", "s0"))
    y, S = kda_chunk(q, k, v, g, decay, s0)
    h = w.T // 2
    y1, S1 = kda_chunk(q[:, :, :h], k[:, :, :h], v[:, :, :h], g[:, :, :h], decay, s0)
    y2, S2 = kda_chunk(q[:, :, h:], k[:, :, h:], v[:, :, h:], g[:, :, h:], decay, S1)
    assert max_rel(torch.cat([y1, y2], 2).float(), y.float()) <= TOL_LOWP
    assert max_rel(S2, S) <= TOL_STATE


def test_layer_glue_after_the_scan_copies_nothing():
    """The KDA layer (models/kimi_k3.py:99-124) views [B, T, H*Dh] projections
    as [B, H, T, Dh], scales the scan output per head and returns
    ``o.transpose(1, 2).contiguous()``.  The scan writes y in its inputs' memory
    order ([B, T, H, Dh]), so the head scale keeps that order and the final
    ``contiguous()`` is a no-op instead of a full copy of y."""
    B, T, H, Dh = 2, 256, 4, 64
    g = torch.Generator().manual_seed(7)
    proj = [torch.randn(B, T, H * Dh, generator=g).to(torch.bfloat16).to(DEV) for _ in range(4)]
    q, k, v, gate = (p.view(B, T, H, Dh).transpose(1, 2) for p in proj)
    o = kda_chunked_scan(q, k, v, gate=gate, decay=0.97, chunk_size=64)
    assert o.stride() == q.stride()
    head_scale = torch.rand(H, device=DEV)
    o = o * head_scale.view(1, H, 1, 1).to(o.dtype)
    t = o.transpose(1, 2)
    assert t.is_contiguous()
    assert t.contiguous().data_ptr() == o.data_ptr()


def test_kernel_trace_times_each_kernel_of_a_step():
    """The library's own CUDA-event tracer names and times every kernel launch."""
    from simpletrain_b200._ffi import KernelTrace
    inp = make_inputs(custom(4, 10, 1024, 128), seed=1, device=DEV)
    q, k, v, g, dy = (inp[n] for n in ("q", "k", "v", "g", "dy"))
    dec = inp["decay"].expand(4, 10, 128)
    with torch.inference_mode(), KernelTrace(64) as tr:
        for _ in range(3):
            torch.ops.kda_b200.chunk_fwd(q, k, v, g, dec, 0.0, None, 64, 0, True)
            torch.ops.kda_b200.chunk_bwd(q, k, v, g, dy, dec, 0.0, None, None, None, 64, 0, True, False)
        torch.cuda.synchronize()
    main = ("fwd_tc_kernel", "bwd_fwddir_tc_kernel", "bwd_revdir_tc_kernel")
    names = [n for n, _ in tr.launches if n in main]
    assert names == list(main) * 3
    # 40 streams on 148 CTA slots are cut into ranges inside streams: the range
    # aggregates and entry folds of the long-stream schedule run too
    assert {n for n, _ in tr.launches} <= set(main) | {"agg_tc_kernel", "entry_fold_kernel"}
    per = tr.per_kernel()
    assert all(per[n][0] == 3 and 0.0 < per[n][1] < 100.0 for n in main)


_BAD_CALLS = r"""
import sys, torch
import simpletrain_b200.ops  # noqa: F401
q = torch.zeros(1, 2, 64, 128, device="cuda", dtype=torch.bfloat16)
for args in ((q, q, q, None, None, 0.9, None, 64, 7, True),      # no such mode
             (q, q, q, None, None, 0.01, None, 64, 2, True)):    # per-step decay below 0.125: the ABI refuses
    try:
        torch.ops.kda_b200.chunk_fwd(*args)
        print("no error")
    except RuntimeError as e:
        print("raised", str(e).splitlines()[0])
"""


def test_op_argument_errors_raise_instead_of_crashing():
    """Errors found in the C++ op (or reported by the C ABI) reach Python as
    RuntimeError with the status text; run in a child process so a crash
    cannot take the test session with it."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", _BAD_CALLS], cwd=root, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    assert len(lines) == 2, out.stdout
    assert lines[0].startswith("raised mode must be") and lines[0].endswith("got 7")
    assert lines[1].startswith("raised kda_fwd_sm100 failed: unsupported configuration") and "(status 3)" in lines[1]
