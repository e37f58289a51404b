"""Per-step (docstring) decay semantics on the sm_100a kernels.

The recurrence of kernels/kda_kernel.py:8-11 (and its never-launched Triton
kernel, :134-180): s_t = a s_{t-1} + k_t^T v_t, y_t = g_t * (q_t s_t), one
decay a per (batch, head).  Small cases are checked against the per-token
recurrence itself (float64, autograd for the gradients); long streams, where
the carry crosses chains of work ranges through precomputed aggregates,
against the float64 chunked restatement, which the CPU tests pin to the
recurrence.

Tolerances: bf16 outputs and gradients within normwise max-rel 2e-2, as for
the chunk-constant mode; the fp32 final state within 5e-3 instead of 1e-3,
because the row-scaled k operand of the state update is rounded to bf16
(relative 2^-9 per element) while the chunk-constant update multiplies the
bf16 inputs exactly -- the same order as the reference kernel's own bf16
store of its final state (kernels/kda_kernel.py:183-189).
"""
import pytest
import torch

from oracle.kda_oracle import max_rel, per_step_chunk_scan, per_step_manual_backward, per_step_recurrence
from simpletrain_b200 import device_status, kda_chunk
from simpletrain_b200 import kda_kernel as dropin

pytestmark = pytest.mark.gpu

TOL_LOWP = 2e-2
TOL_STATE = 5e-3
DEV = "cuda"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert device_status() == 0, "a device-side bounded wait expired"


def _rand(B, H, T, D, seed, gate=True, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)

    def bthd(x):
        return x.to(dtype).transpose(1, 2)

    q = bthd(torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1))
    k = bthd(torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1))
    v = bthd(torch.randn(B, T, H, D, generator=g))
    gt = bthd(torch.sigmoid(torch.randn(B, T, H, D, generator=g))) if gate else None
    dy = bthd(torch.randn(B, T, H, D, generator=g))
    heads = torch.sigmoid(torch.randn(H, generator=g) + 3.0)   # per-head decays in (0.5, 1)
    return q, k, v, gt, dy, heads


def _decay(kind, heads):
    return heads if kind == "head" else float(kind)


def oracle_recurrence(q, k, v, g, decay, s0, dy=None, dsT=None):
    """float64 per-token recurrence, autograd for the gradients."""
    leaves = [t.detach().cpu().double().requires_grad_(dy is not None) for t in (q, k, v)]
    gl = g.detach().cpu().double().requires_grad_(dy is not None) if g is not None else None
    sl = s0.detach().cpu().double().requires_grad_(dy is not None) if s0 is not None else None
    dec = decay.double() if torch.is_tensor(decay) else decay
    y, S = per_step_recurrence(*leaves, gl, dec, sl)
    out = {"y": y.detach(), "S": S.detach()}
    if dy is not None:
        loss = (y * dy.cpu().double()).sum()
        if dsT is not None:
            loss = loss + (S * dsT.double()).sum()
        loss.backward()
        out.update(dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad)
        if gl is not None:
            out["dg"] = gl.grad
        if sl is not None:
            out["ds0"] = sl.grad
    return out


def oracle_chunked(q, k, v, g, decay, s0, dy, dsT):
    """float64 chunked restatement and its explicit backward (long streams)."""
    f = lambda t: t.cpu().double() if t is not None else None
    dec = decay.double() if torch.is_tensor(decay) else decay
    y, S = per_step_chunk_scan(f(q), f(k), f(v), f(g), dec, 64, f(s0))
    dq, dk, dv, dg, ds0 = per_step_manual_backward(f(q), f(k), f(v), f(g), dec, 64, f(s0), f(dy), f(dsT))
    out = {"y": y, "S": S, "dq": dq, "dk": dk, "dv": dv}
    if g is not None:
        out["dg"] = dg
    if s0 is not None:
        out["ds0"] = ds0
    return out


def run_gpu(q, k, v, g, decay, s0, dy=None, dsT=None):
    grad = dy is not None
    leaves = [t.detach().to(DEV).requires_grad_(grad) for t in (q, k, v)]
    gl = g.detach().to(DEV).requires_grad_(grad) if g is not None else None
    sl = s0.detach().to(DEV).requires_grad_(grad) if s0 is not None else None
    dec = decay.to(DEV) if torch.is_tensor(decay) else decay
    y, S = kda_chunk(*leaves, gl, dec, sl, 64, per_step=True)
    out = {"y": y.detach(), "S": S.detach()}
    if grad:
        loss = (y.float() * dy.to(DEV).float()).sum()
        if dsT is not None:
            loss = loss + (S * dsT.to(DEV)).sum()
        loss.backward()
        out.update(dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad)
        if gl is not None:
            out["dg"] = gl.grad
        if sl is not None:
            out["ds0"] = sl.grad
    return out


def compare(got, ref):
    errs = {}
    for key in ref:
        tol = TOL_STATE if key == "S" else TOL_LOWP
        errs[key] = max_rel(got[key].double().cpu(), ref[key])
        assert errs[key] <= tol, f"{key}: max_rel {errs[key]:.3e} > {tol:.0e}  (all: {errs})"
    return errs


SMALL = [
    # B, H, T, D, gate, decay, s0
    (2, 3, 256, 64, True, "0.9", False),
    (1, 2, 200, 128, True, "head", True),
    (2, 2, 130, 64, False, "0.5", True),
    (1, 1, 1, 64, True, "0.97", True),
    (1, 2, 77, 128, False, "0.125", True),     # the smallest decay the row scaling takes
    (1, 2, 200, 64, True, "0.2", True),        # a^64 below fp32's range, four chunks carried in one range
    (1, 2, 192, 128, True, "1.0", False),      # no decay: plain causal linear attention
]


@pytest.mark.parametrize("B,H,T,D,gate,dkind,with_s0", SMALL)
def test_per_step_forward_backward_small(B, H, T, D, gate, dkind, with_s0):
    q, k, v, g, dy, heads = _rand(B, H, T, D, seed=11, gate=gate)
    decay = _decay(dkind, heads)
    s0 = torch.randn(B, H, D, D) * 0.05 if with_s0 else None
    dsT = torch.randn(B, H, D, D) * 0.1
    compare(run_gpu(q, k, v, g, decay, s0, dy, dsT), oracle_recurrence(q, k, v, g, decay, s0, dy, dsT))


def test_per_step_fp16_inputs():
    q, k, v, g, dy, _ = _rand(1, 2, 160, 128, seed=16, dtype=torch.float16)
    s0 = torch.randn(1, 2, 128, 128) * 0.05
    dsT = torch.randn(1, 2, 128, 128) * 0.1
    got = run_gpu(q, k, v, g, 0.93, s0, dy, dsT)
    assert got["y"].dtype == torch.float16
    compare(got, oracle_recurrence(q, k, v, g, 0.93, s0, dy, dsT))


LONG = [
    (1, 1, 4096, 128, True, "0.999", True),
    (1, 2, 3000, 64, True, "head", False),
    (2, 1, 2500, 128, False, "0.99", True),
]


@pytest.mark.parametrize("B,H,T,D,gate,dkind,with_s0", LONG)
def test_per_step_long_streams(B, H, T, D, gate, dkind, with_s0):
    q, k, v, g, dy, heads = _rand(B, H, T, D, seed=12, gate=gate)
    decay = _decay(dkind, heads)
    s0 = torch.randn(B, H, D, D) * 0.02 if with_s0 else None
    dsT = torch.randn(B, H, D, D) * 0.1
    compare(run_gpu(q, k, v, g, decay, s0, dy, dsT), oracle_chunked(q, k, v, g, decay, s0, dy, dsT))


def test_per_step_split_consistency():
    """Size-independent: [0, T/2) then [T/2, T) from the handed-over state equals one scan."""
    q, k, v, g, _, heads = _rand(2, 4, 4096, 128, seed=13)
    q, k, v, g = (t.to(DEV) for t in (q, k, v, g))
    dec = heads.to(DEV)
    y, S = kda_chunk(q, k, v, g, dec, None, per_step=True)
    h = 2048 + 32   # not a chunk multiple: the first half ends with a ragged chunk
    y1, S1 = kda_chunk(q[:, :, :h], k[:, :, :h], v[:, :, :h], g[:, :, :h], dec, None, per_step=True)
    y2, S2 = kda_chunk(q[:, :, h:], k[:, :, h:], v[:, :, h:], g[:, :, h:], dec, S1, per_step=True)
    assert max_rel(torch.cat([y1, y2], 2).float(), y.float()) <= TOL_LOWP
    assert max_rel(S2, S) <= TOL_STATE


def test_per_step_differs_from_chunk_constant():
    """The two semantics agree only when nothing decays."""
    q, k, v, g, _, _ = _rand(1, 2, 256, 64, seed=14)
    q, k, v, g = (t.to(DEV) for t in (q, k, v, g))
    y_ps, _ = kda_chunk(q, k, v, g, 0.9, None, per_step=True)
    y_cc, _ = kda_chunk(q, k, v, g, 0.9, None)
    assert max_rel(y_ps.float(), y_cc.float()) > 0.1
    y_ps1, _ = kda_chunk(q, k, v, g, 1.0, None, per_step=True)
    y_cc1, _ = kda_chunk(q, k, v, g, 1.0, None)
    assert max_rel(y_ps1.float(), y_cc1.float()) <= TOL_LOWP


def test_per_step_dropin_semantics(monkeypatch):
    """kernels.kda_kernel with SEMANTICS = "per_step" runs the docstring recurrence."""
    q, k, v, g, _, _ = _rand(1, 2, 128, 64, seed=15)
    monkeypatch.setattr(dropin, "SEMANTICS", "per_step")
    y = dropin.kda_chunked_scan(q.to(DEV), k.to(DEV), v.to(DEV), gate=g.to(DEV), decay=0.95, chunk_size=64)
    ref = oracle_recurrence(q, k, v, g, 0.95, None)
    assert max_rel(y.double().cpu(), ref["y"]) <= TOL_LOWP


@pytest.mark.parametrize("decay,exc,dtype", [
    (0.05, ValueError, torch.bfloat16),                   # below the supported range
    (1.5, ValueError, torch.bfloat16),
    (0.8, ValueError, torch.float16),                     # fp16 takes [0.9, 1]
    (torch.full((2, 64), 0.9), ValueError, torch.bfloat16),  # per key channel: not one per head
])
def test_per_step_rejects_unsupported_decay(decay, exc, dtype):
    q = torch.randn(1, 2, 64, 64, device=DEV, dtype=dtype)
    d = decay.to(DEV) if torch.is_tensor(decay) else decay
    with pytest.raises(exc):
        kda_chunk(q, q, q, None, d, None, per_step=True)


def test_per_step_decay_is_not_differentiated():
    q = torch.randn(1, 2, 64, 64, device=DEV, dtype=torch.bfloat16)
    d = torch.full((2,), 0.9, device=DEV, requires_grad=True)
    with pytest.raises(NotImplementedError):
        kda_chunk(q, q, q, None, d, None, per_step=True)
    with pytest.raises(ValueError):
        kda_chunk(q, q, q, None, 0.9, None, reference_exact=True, per_step=True)
