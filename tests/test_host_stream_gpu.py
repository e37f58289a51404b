"""HostScan: host tensors streamed through the GPU in batch slices.

The slices are independent (batch) rows, so the results must equal the scan
of the whole batch on the device (kda_chunk + autograd): outputs and the
per-row gradients bit for bit up to the fp32 summation order of the range
schedule, which differs between a slice and the whole batch: normwise
max-rel 8e-3 on the bf16/fp16 tensors (a rounding step of the largest
element is up to 2^-7 of it in bf16), 1e-4 on the fp32 states and the decay
gradient summed over the batch.
"""
import pytest
import torch

from oracle.kda_oracle import max_rel
from simpletrain_b200 import device_status, kda_chunk
from simpletrain_b200.host_stream import HostScan

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert device_status() == 0, "a device-side bounded wait expired"


def _inputs(B, H, T, D, seed, dtype=torch.bfloat16, gate=True):
    g = torch.Generator().manual_seed(seed)

    def host(x):  # [B, T, H, D] pinned memory viewed [B, H, T, D]
        p = torch.empty(B, T, H, D, dtype=dtype, pin_memory=True)
        p.copy_(x)
        return p.transpose(1, 2)

    q = host(torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1))
    k = host(torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1))
    v = host(torch.randn(B, T, H, D, generator=g))
    gt = host(torch.sigmoid(torch.randn(B, T, H, D, generator=g))) if gate else None
    dy = host(torch.randn(B, T, H, D, generator=g))
    return q, k, v, gt, dy, g


def _device_reference(q, k, v, g, decay, dy, s0, per_step=False):
    leaves = [t.to(DEV).requires_grad_(dy is not None) for t in (q, k, v)]
    gl = g.to(DEV).requires_grad_(dy is not None) if g is not None else None
    dl = decay.to(DEV).requires_grad_(dy is not None and not per_step) if torch.is_tensor(decay) else decay
    sl = s0.to(DEV).requires_grad_(dy is not None) if s0 is not None else None
    y, S = kda_chunk(*leaves, gl, dl, sl, 64, per_step=per_step)
    out = {"y": y.detach(), "final_state": S.detach()}
    if dy is not None:
        wrt = leaves + ([gl] if gl is not None else []) + ([dl] if torch.is_tensor(dl) and dl.requires_grad else []) \
            + ([sl] if sl is not None else [])
        grads = torch.autograd.grad([y], wrt, [dy.to(DEV)])
        names = ["dq", "dk", "dv"] + (["dg"] if gl is not None else []) \
            + (["ddecay"] if torch.is_tensor(dl) and dl.requires_grad else []) + (["ds0"] if sl is not None else [])
        out.update(zip(names, grads))
    return out


def _check(got, ref):
    assert set(got) == set(ref), (sorted(got), sorted(ref))
    for n, r in ref.items():
        assert got[n].device.type == "cpu" and got[n].shape == r.shape, n
        tol = 8e-3 if r.dtype in (torch.bfloat16, torch.float16) else 1e-4
        e = max_rel(got[n].double(), r.double().cpu())
        assert e <= tol, f"{n}: max_rel {e:.2e} > {tol:.0e}"


@pytest.mark.parametrize("B,H,T,D,slices,dshape", [
    (5, 3, 200, 64, 2, "HD"),     # ragged slices (2, 3 rows), ragged last chunk
    (4, 2, 256, 128, 4, "H"),     # one row per slice, per-head decay
    (3, 2, 130, 128, None, "HD"),  # default slicing
])
def test_host_scan_fwd_bwd_matches_device(B, H, T, D, slices, dshape):
    q, k, v, g, dy, gen = _inputs(B, H, T, D, seed=21)
    decay = torch.sigmoid(torch.randn(H, D, generator=gen) + 3.0)
    if dshape == "H":
        decay = decay[:, 0].contiguous()
    s0 = torch.randn(B, H, D, D, generator=gen) * 0.05
    got = HostScan(DEV, slices=slices)(q, k, v, g, decay, dy=dy, initial_state=s0)
    _check(got, _device_reference(q, k, v, g, decay, dy, s0))


def test_host_scan_forward_only_float_decay():
    q, k, v, _, _, _ = _inputs(6, 2, 300, 64, seed=22, gate=False)
    got = HostScan(DEV, slices=3)(q, k, v, None, 0.97)
    _check(got, _device_reference(q, k, v, None, 0.97, None, None))


def test_host_scan_per_step_fp16():
    q, k, v, g, dy, gen = _inputs(4, 2, 192, 128, seed=23, dtype=torch.float16)
    decay = torch.tensor([0.95, 0.99])
    got = HostScan(DEV, slices=2, per_step=True)(q, k, v, g, decay, dy=dy)
    _check(got, _device_reference(q, k, v, g, decay, dy, None, per_step=True))


def test_host_scan_reuses_buffers_and_new_shapes():
    scan = HostScan(DEV, slices=2)
    q, k, v, g, dy, _ = _inputs(2, 2, 128, 64, seed=24)
    a = scan(q, k, v, g, 0.9, dy=dy)
    ptr = a["y"].data_ptr()
    ref = {n: t.clone() for n, t in a.items()}
    b = scan(q, k, v, g, 0.9, dy=dy)        # the second result-buffer set
    c = scan(q, k, v, g, 0.9, dy=dy)        # the first one again
    assert b["y"].data_ptr() != ptr and c["y"].data_ptr() == ptr
    for n in ref:
        assert torch.equal(b[n], ref[n]) and torch.equal(c[n], ref[n]), n   # same inputs and slices: identical
    b["dq"].add_(1)   # ordinary tensors: in-place use outside inference mode works
    q2, k2, v2, g2, dy2, _ = _inputs(3, 2, 64, 64, seed=25)
    c = scan(q2, k2, v2, g2, 0.9, dy=dy2)
    _check(c, _device_reference(q2, k2, v2, g2, 0.9, dy2, None))


def test_host_scan_submitted_calls_overlap_and_keep_their_results():
    """Calls queued with submit() before waiting: each gets its own inputs' results."""
    scan = HostScan(DEV, slices=4)
    batches = [_inputs(4, 2, 192, 128, seed=30 + i) for i in range(4)]
    decay = torch.sigmoid(torch.randn(2, 128, generator=torch.Generator().manual_seed(3)) + 3.0)
    pend, got = None, []
    for q, k, v, g, dy, _ in batches:
        p = scan.submit(q, k, v, g, decay, dy=dy)
        if pend is not None:
            got.append({n: t.clone() for n, t in pend.wait().items()})
        pend = p
    got.append({n: t.clone() for n, t in pend.wait().items()})
    for (q, k, v, g, dy, _), res in zip(batches, got):
        _check(res, _device_reference(q, k, v, g, decay, dy, None))


def _pinned_copy(t):
    if not torch.is_tensor(t):
        return t
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h


@pytest.mark.parametrize("sets,lag", [(2, 1), (3, 2)])
def test_sharded_host_scan_pipelined_steps(sets, lag):
    """ShardedHostScan (one rank): consecutive steps with different inputs, each
    step submitted before step i-lag's results are read -- the pattern bench.py's
    end-to-end number uses with three buffer sets -- give every step the results
    of the same scan run directly on the device."""
    from simpletrain_b200.host_stream import ShardedHostScan
    from simpletrain_b200.sharding import ShardedScan

    B, H, T, D = 2, 4, 700, 128
    decay = torch.sigmoid(torch.randn(H, D, generator=torch.Generator().manual_seed(3)) + 3.0)
    steps = 5
    data = [_inputs(B, H, T, D, seed=40 + i) for i in range(steps)]
    sc = ShardedScan(B, H, T, D, 64, 1, 0)
    runner = ShardedHostScan(sc, DEV, True, False, sets=sets)
    hosts = []
    for q, k, v, g, dy, _ in data:
        pieces = sc.load({"q": q, "k": k, "v": v, "g": g, "dy": dy, "decay": decay, "s0": None})
        hosts.append([{n: _pinned_copy(t) for n, t in p.items()} for p in pieces])
    pend, got = [], []
    for i in range(steps + lag):
        if i < steps:
            pend.append(runner.submit(hosts[i]))
        if i >= lag:
            res = pend[i - lag].wait()
            got.append({n: t.clone() for n, t in res[0].items()})
    assert len(got) == steps
    for (q, k, v, g, dy, _), out in zip(data, got):
        ref = _device_reference(q, k, v, g, decay, dy, None)
        for n in ("y", "final_state", "dq", "dk", "dv", "dg"):
            tol = 1e-4 if n == "final_state" else 8e-3
            e = max_rel(out[n].float(), ref[n].float().cpu())
            assert e <= tol, (n, e)
        e = max_rel(out["ddecay"].float().sum(0).reshape(H, D), ref["ddecay"].float().cpu().reshape(H, D))
        assert e <= 1e-4, ("ddecay", e)
