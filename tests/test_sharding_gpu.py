"""The sharded scan on the CUDA kernels, with every rank emulated in one process
on one GPU, and the ops captured in a CUDA graph.

``ShardedScan``'s phases are driven rank by rank: every rank's local pieces,
then the exchange (the ranks' tiles stacked, as all_gather would give them),
then every rank's remaining piece -- the same calls and the same data the ranks
of a multi-GPU run make, without a collective.  The assembled result is
compared with one unsharded run on the same GPU and, on the streams that are
split in time, with the CPU oracle.
"""
import pytest
import torch

from oracle.kda_oracle import chunk_scan, decay_bhd1, max_rel
from simpletrain_b200 import device_status
from simpletrain_b200.sharding import ShardedScan, cuda_scan_fns
from simpletrain_b200.workloads import custom, make_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert device_status() == 0, "a device-side bounded wait expired"


def _emulate(B, H, T, D, world, inp, decay, balance="chunks"):
    fwd, bwd = cuda_scan_fns(64, 0)
    scans = [ShardedScan(B, H, T, D, 64, world, r, fwd=fwd, bwd=bwd, balance=balance) for r in range(world)]
    xs = [sc.load(dict(inp, decay=decay)) for sc in scans]
    with torch.inference_mode():
        outs = [sc.forward_local(x) for sc, x in zip(scans, xs)]
        tiles = torch.stack([sc.forward_exit(x, o) for sc, x, o in zip(scans, xs, outs)]) if scans[0].split else None
        outs = [sc.forward_rest(x, o, tiles) for sc, x, o in zip(scans, xs, outs)]
        grads = [sc.backward_local(x, True, inp["s0"] is not None) for sc, x in zip(scans, xs)]
        tiles = torch.stack([sc.backward_entry(x, g) for sc, x, g in zip(scans, xs, grads)]) if scans[0].split \
            else None
        grads = [sc.backward_rest(x, g, tiles) for sc, x, g in zip(scans, xs, grads)]
    f32 = torch.float32
    shapes = {n: ((B, H, T, D), torch.bfloat16) for n in ("y", "dq", "dk", "dv", "dg")}
    shapes.update(final_state=((B, H, D, D), f32), ddecay=((B, H, D), f32))
    if inp["s0"] is not None:
        shapes["ds0"] = ((B, H, D, D), f32)
    total = None
    for sc, o, g in zip(scans, outs, grads):
        part = sc.assemble([dict(a, **b) for a, b in zip(o, g)], shapes, DEV, reduce=False)
        total = part if total is None else {n: total[n] + part[n] for n in total}
    return scans, total


def _unsharded(B, H, T, D, inp, decay):
    return _emulate(B, H, T, D, 1, inp, decay)[1]


@pytest.mark.parametrize("B,H,T,world", [
    (1, 28, 2048, 8),     # the 10b head count over 8 ranks: four streams split in half
    (1, 7, 640, 4),       # 70 chunks over 4 ranks: splits at uneven chunk positions
    (2, 3, 1000, 4),      # ragged last chunk, pieces across batch rows
    (2, 8, 512, 4),       # whole streams only: no exchange
])
def test_emulated_ranks_match_one_gpu_and_the_oracle(B, H, T, world):
    D = 128
    inp = make_inputs(custom(B, H, T, D, s0_std=0.02, decay_mean=4.0), seed=5, device=DEV)
    decay = inp["decay"]
    scans, got = _emulate(B, H, T, D, world, inp, decay)
    ref = _unsharded(B, H, T, D, inp, decay)
    for n in got:
        tol = 1e-3 if n == "final_state" else 2e-2
        e = max_rel(got[n].float().cpu(), ref[n].float().cpu())
        assert e <= tol, (n, e)
    split = sorted({p.s0 for sc in scans for p in sc.pieces if not p.whole})
    assert bool(split) == scans[0].split
    # the streams split in time, against the oracle (fp32, CPU)
    for s in split[:2]:
        b, h = divmod(s, H)
        leaves = {n: inp[n][b:b + 1, h:h + 1].detach().cpu().float().requires_grad_(True)
                  for n in ("q", "k", "v", "g")}
        dl = decay[h:h + 1].detach().cpu().float().requires_grad_(True)
        s0 = inp["s0"][b:b + 1, h:h + 1].detach().cpu().float().requires_grad_(True)
        y, S = chunk_scan(leaves["q"], leaves["k"], leaves["v"], leaves["g"], decay_bhd1(dl, 1, 1, D), 64,
                          initial_state=s0)
        dy = inp["dy"][b:b + 1, h:h + 1].cpu().float()
        gr = torch.autograd.grad((y * dy).sum(), [leaves[n] for n in ("q", "k", "v", "g")] + [dl, s0])
        pairs = {"y": (got["y"], y), "final_state": (got["final_state"], S), "dq": (got["dq"], gr[0]),
                 "dk": (got["dk"], gr[1]), "dv": (got["dv"], gr[2]), "dg": (got["dg"], gr[3]),
                 "ds0": (got["ds0"], gr[5])}
        for n, (a, r) in pairs.items():
            tol = 1e-3 if n == "final_state" else 2e-2     # gradients (ds0 too) come from bf16 operands
            e = max_rel(a[b:b + 1, h:h + 1].float().cpu(), r)
            assert e <= tol, (s, n, e)
        e = max_rel(got["ddecay"][b, h].cpu(), gr[4][0])
        assert e <= 2e-2, (s, "ddecay", e)


@pytest.mark.parametrize("B,H,T,world", [
    (1, 28, 2048, 8),     # the 10b head count over 8 ranks: 4, 4, 4, 4, 3, 3, 3, 3 whole streams
    (2, 5, 700, 4),       # 3, 3, 2, 2 streams, runs across batch rows (copied), ragged last chunk
])
def test_whole_stream_shards_match_one_gpu(B, H, T, world):
    D = 128
    inp = make_inputs(custom(B, H, T, D, s0_std=0.02, decay_mean=4.0), seed=6, device=DEV)
    scans, got = _emulate(B, H, T, D, world, inp, inp["decay"], balance="streams")
    assert not scans[0].split and all(p.whole for sc in scans for p in sc.pieces)
    ref = _unsharded(B, H, T, D, inp, inp["decay"])
    for n in got:
        tol = 1e-3 if n == "final_state" else 2e-2
        e = max_rel(got[n].float().cpu(), ref[n].float().cpu())
        assert e <= tol, (n, e)


def test_forward_and_backward_replay_in_a_cuda_graph():
    """The ops allocate from the caching allocator and run on the current stream,
    so a fwd+bwd step captures into a CUDA graph; replays match the eager step."""
    B, H, T, D = 2, 10, 1024, 128
    inp = make_inputs(custom(B, H, T, D), seed=9, device=DEV)
    q, k, v, g, dy = (inp[n] for n in ("q", "k", "v", "g", "dy"))
    dec = inp["decay"].expand(B, H, D)

    def step():
        y, S = torch.ops.kda_b200.chunk_fwd(q, k, v, g, dec, 0.0, None, 64, 0, True)
        grads = torch.ops.kda_b200.chunk_bwd(q, k, v, g, dy, dec, 0.0, None, None, None, 64, 0, True, False)
        return (y, S) + tuple(grads[:5])

    with torch.inference_mode():
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                eager = step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
    for a, b in zip(out, eager):
        assert torch.equal(a, b)


def test_kernel_trace_inside_a_cuda_graph():
    """The tracer brackets captured launches with event nodes: after each replay
    it reads that replay's per-kernel device times."""
    from simpletrain_b200._ffi import KernelTrace
    B, H, T, D = 4, 10, 1024, 128
    inp = make_inputs(custom(B, H, T, D), seed=2, device=DEV)
    q, k, v, g, dy = (inp[n] for n in ("q", "k", "v", "g", "dy"))
    dec = inp["decay"].expand(B, H, D)

    def step():
        torch.ops.kda_b200.chunk_fwd(q, k, v, g, dec, 0.0, None, 64, 0, True)
        torch.ops.kda_b200.chunk_bwd(q, k, v, g, dy, dec, 0.0, None, None, None, 64, 0, True, False)

    with torch.inference_mode():
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with KernelTrace(64) as tr:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            per_replay = []
            for _ in range(3):
                graph.replay()
                torch.cuda.synchronize()
                per_replay.append(tr.read())
            del graph
    main = ("fwd_tc_kernel", "bwd_fwddir_tc_kernel", "bwd_revdir_tc_kernel")
    for got in per_replay:
        names = [n for n, _ in got if n in main]
        assert names == list(main)
        assert all(0.0 < ms < 100.0 for _, ms in got)
    assert len(tr.launches) == sum(len(r) for r in per_replay)
