#!/usr/bin/env python
"""KDA chunked-scan throughput on B200: forward + backward tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload 1b-fwdbwd]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)
    python bench.py --impl reference ...                     (CPU arm)

One step = one forward + backward pass of the KDA scan over one batch of the
workload (default: the 1b-variant shape B=16, H=10, T=2048, D=128, chunk 64,
bf16).  With N ranks the one global problem is sharded (``--scaling strong``,
the default; ``simpletrain_b200.sharding``): each rank takes a run of whole
streams (``--balance streams``, the default; no communication on the data
path), or (``--balance chunks``) an exactly balanced range of the
stream-major (stream, chunk) sequence, where a stream that straddles two
ranks is split in time with one small all_gather of carried states per
direction.  ``value`` = the problem's tokens / the max-over-ranks device time
per step.
``--scaling weak`` gives every rank its own full batch instead.

Each rank's step is captured once in a CUDA graph and replayed (the step's
launches cost more host time than a rank's share of the work takes on the
device at 8 GPUs).  Per-kernel device times come from the library's own
CUDA-event tracer (``kda_trace_start``): the step is captured once more with
the tracer on, which brackets every kernel with event nodes of the graph, and
replayed right after the timed region.  At N > 1 the ranks' results are
gathered on rank 0 after timing and checked against a single-GPU run of the
whole problem.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

from simpletrain_b200.workloads import WORKLOADS, make_inputs  # noqa: E402

METRIC = "KDA fwd+bwd tokens/s"
UNIT = "tokens/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
DATA = ("synthetic (seeded; q,k L2-normalised N(0,1), v N(0,1), g sigmoid(N(0,1)), "
        "decay sigmoid(N(3,1)) per key channel (N(4,1) at 10b, with an N(0,0.02) initial state))")

# Algorithmic HBM bytes of each kernel per token-head, in units of D x element
# size: the tensors it must read and write once.  fwd: q,k,v,g in, y out; the
# backward's forward-direction pass: q,k,v,g,dy in, dq,dg and dO = dy*g (handed
# to the second pass) out; its reverse pass: q,k,v,dO in, dk,dv out.
KERNEL_BYTES_D = {"fwd_tc_kernel": 5, "bwd_fwddir_tc_kernel": 8, "bwd_revdir_tc_kernel": 6}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


def semantics(args, w):
    """(op mode, decay kind, need d(decay), label) the workload runs in.

    D == chunk (the 100m variant): the reference's own literal K V^T update with
    a float decay, as SimpleTrain's model calls it (models/kimi_k3.py:109-118).
    Otherwise the K^T V update with a per-key-channel decay and its gradient;
    --per-step: the per-token recurrence with one decay per head."""
    if args.per_step:
        return 2, "head", False, "per-step decay (one per head)"
    if w.D == w.chunk and not args.corrected:
        return 1, "float", False, "literal K V^T update (the reference's own at D == chunk), float decay"
    return 0, "channel", w.backward, "K^T V update, chunk-constant per-channel decay (with its gradient)"


def decay_input(kind, decay):
    if kind == "head":
        return decay[:, :1].contiguous()            # [H, 1]: the first channel's, per head
    if kind == "float":
        return float(decay.mean())                  # the model's float(decay.mean())
    return decay                                    # [H, D]


# --------------------------------------------------------------------------- #
# clocks during warm-up and the timed region
# --------------------------------------------------------------------------- #
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            t0 = time.time()
            while os.path.getsize(self.path) == 0 and self.proc.poll() is None and time.time() - t0 < 3.0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            if self.proc.poll() is None:
                self.proc.terminate()
                try:
                    self.proc.wait(timeout=5)
                except Exception:
                    self.proc.kill()
            if not self.fh.closed:
                self.fh.close()

    def summary(self):
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None,
                "covers": "warm-up and timed region"}


# --------------------------------------------------------------------------- #
# our arm
# --------------------------------------------------------------------------- #
def traffic_per_token_head(kernel: str, D: int):
    """DRAM bytes per token-head of one kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as fh:
        ent = json.load(fh).get(f"{kernel}:D{D}")
    return ent["bytes_per_token_head"] if ent else None


def global_inputs(w, dev, rank, world, seed):
    """The seeded global problem on every rank's device: drawn on the host by
    rank 0 (the same bytes the tests use) and broadcast over NCCL."""
    import torch.distributed as dist
    if rank == 0:
        inp = make_inputs(w, seed=seed, device=dev)
    else:
        bthd = (w.B, w.T, w.H, w.D)
        inp = {n: torch.empty(bthd, dtype=w.dtype, device=dev).transpose(1, 2)
               for n in ("q", "k", "v", "g") + (("dy",) if w.backward else ())}
        inp["decay"] = torch.empty(w.H, w.D, dtype=torch.float32, device=dev)
        inp["s0"] = torch.empty(w.B, w.H, w.D, w.D, dtype=torch.float32, device=dev) if w.s0_std > 0 else None
        if not w.backward:
            inp["dy"] = None
    if world > 1:
        for n in ("q", "k", "v", "g", "dy", "decay", "s0"):
            t = inp.get(n)
            if t is not None:
                # [B, H, T, D] views over [B, T, H, D] memory: broadcast the memory
                base = t.transpose(1, 2) if t.dim() == 4 and n != "s0" else t
                dist.broadcast(base, 0)
    return inp


def run_ours(args, w, rank, world, local_rank):
    clk = ClockSampler(local_rank)
    try:
        return _run_ours(args, w, rank, world, local_rank, clk)
    finally:
        clk.__exit__(None, None, None)


def _run_ours(args, w, rank, world, local_rank, clk):
    import torch.distributed as dist

    import simpletrain_b200.ops  # noqa: F401  (loads the ops)
    from simpletrain_b200 import _ffi
    from simpletrain_b200.ops import device_status
    from simpletrain_b200.sharding import ShardedScan, cuda_scan_fns, nccl_exchange

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    strong = args.scaling == "strong"
    mode, dkind, need_dd, sem_label = semantics(args, w)
    clk.__enter__()          # sampled from the warm-up to the end of the timed region

    if strong:
        inp = global_inputs(w, dev, rank, world, seed=0)
    else:
        inp = make_inputs(w, seed=rank, device=dev)
    decay = decay_input(dkind, inp["decay"])
    B, H, T, D = w.B, w.H, w.T, w.D
    fwd, bwd = cuda_scan_fns(w.chunk, mode)
    sworld, srank = (world, rank) if strong else (1, 0)
    sc = ShardedScan(B, H, T, D, w.chunk, sworld, srank, fwd=fwd, bwd=bwd,
                     exchange=nccl_exchange() if sworld > 1 else None, balance=args.balance)
    x = sc.load({"q": inp["q"], "k": inp["k"], "v": inp["v"], "g": inp["g"], "dy": inp["dy"],
                 "decay": decay, "s0": inp["s0"]})
    need_ds0 = inp["s0"] is not None
    rank_token_heads = sum(p.nstreams * (min(T, p.c1 * w.chunk) - p.c0 * w.chunk) for p in sc.pieces)

    def step():
        outs = sc.forward(x)
        grads = sc.backward(x, need_dd, need_ds0) if w.backward else None
        return outs, grads

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (eager, on a side stream as graph capture requires), then capture
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(stream)
    with torch.inference_mode():
        with torch.cuda.stream(side):
            for _ in range(max(args.warmup, 1)):
                step()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = None
        if not args.eager:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            run = graph.replay
        else:
            run = step
        for _ in range(2):
            run()
        torch.cuda.synchronize()

    steps = args.steps
    if steps is None:
        t0 = time.perf_counter()
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        per = (time.perf_counter() - t0) / 3
        steps = int(min(5000, max(10, 3.0 / max(per, 1e-6))))
        if world > 1:
            t = torch.tensor([steps], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            steps = int(t.item())

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _ffi.launch_count()
    barrier()
    torch.cuda.synchronize()
    with torch.inference_mode():
        start.record(stream)
        for _ in range(steps):
            run()
        end.record(stream)
        torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    barrier()
    ms = start.elapsed_time(end)
    graphed_launches = _ffi.launch_count() - launches0   # launches issued from the host (0 when replayed)

    # ---- per-kernel device times: the library's event tracer ----------------------
    # (graph mode: the step captured once more with the tracer on, so each launch
    # is bracketed by event nodes of the graph; the times are read after every replay)
    trace_steps = min(steps, 50 if graph is None else 20)
    with torch.inference_mode():
        barrier()
        with _ffi.KernelTrace(max_launches=16 * trace_steps + 16) as tr:
            if graph is not None:
                traced = torch.cuda.CUDAGraph()
                with torch.cuda.graph(traced):
                    step()
                for _ in range(trace_steps):
                    traced.replay()
                    torch.cuda.synchronize()
                    tr.read()
                del traced
            else:
                for _ in range(trace_steps):
                    step()
                torch.cuda.synchronize()
        barrier()
    per_kernel = tr.per_kernel()
    kernels_per_step = sum(c for c, _ in per_kernel.values()) / trace_steps
    launches = graphed_launches if graph is None else int(round(kernels_per_step * steps))

    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    status = device_status(dev)
    if status:
        raise RuntimeError(f"device-side KDA status {status}")

    tokens_per_step = (B * T) if strong else world * B * T
    value = tokens_per_step * steps / (ms / 1e3)

    # ---- roofline of the dominant kernel -----------------------------------------
    peaks = load_peaks()
    esz = torch.finfo(w.dtype).bits // 8
    kernels = {}
    for name, (count, mean_ms) in sorted(per_kernel.items()):
        ent = {"launches_per_step": round(count / trace_steps, 3), "ms": round(mean_ms, 5),
               "share": round(count * mean_ms / sum(c * m for c, m in per_kernel.values()), 4)}
        if name in KERNEL_BYTES_D:
            nbytes = rank_token_heads * KERNEL_BYTES_D[name] * D * esz
            ent["algorithmic_bytes"] = nbytes
            ent["GB_s"] = round(nbytes / (mean_ms / 1e3) / 1e9, 1)
            ent["frac_hbm"] = round(nbytes / (mean_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)
        kernels[name] = ent
    dom = max(per_kernel, key=lambda n: per_kernel[n][0] * per_kernel[n][1])
    dbytes = kernels[dom].get("algorithmic_bytes")
    dms = per_kernel[dom][1]
    tph = traffic_per_token_head(dom, D)
    step_bytes = rank_token_heads * (14 if w.backward else 5) * D * esz     # q,k,v,g,y (+dy,dq,dk,dv,dg)
    step_flops = rank_token_heads * ((12 if w.backward else 4) * w.chunk * D + (12 if w.backward else 4) * D * D)
    per_step_s = ms / steps / 1e3
    roofline = {"bound": "hbm", "kernel": dom,
                "achieved": round(dbytes / (dms / 1e3) / 1e9, 1) if dbytes else None,
                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(dbytes / (dms / 1e3) / 1e9 / peaks["hbm_gbs"], 4) if dbytes else None,
                "traffic": round(tph * rank_token_heads) if tph else None,
                "algorithmic_bytes": dbytes, "peak_source": peaks["source"],
                "kernel_ms": round(dms, 5),
                "kernel_times": (f"CUDA events around each launch (library tracer), {trace_steps} "
                                 + ("replays of the step captured as a CUDA graph with event nodes"
                                    if graph is not None else "eager steps")
                                 + " right after the timed region"),
                "step_frac_hbm": round(step_bytes / per_step_s / 1e9 / peaks["hbm_gbs"], 4),
                "step_frac_tensor": round(step_flops / per_step_s / 1e12 / peaks["bf16_tflops"], 4),
                "step_bytes_per_rank": step_bytes}

    # ---- the sharded result against one GPU's ------------------------------------
    check = run_check(args, w, sc, x, inp, decay, mode, need_dd, rank, world, dev) if strong and world > 1 else None

    # ---- end to end through the host-buffer API ----------------------------------
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, w, sc, x, rank, world, dev, need_dd, need_ds0, tokens_per_step)

    # ---- CPU baseline (rank 0, N = 1) ----------------------------------------------
    cpu = None
    if args.per_step:
        cpu = {"unavailable": "the reference has no CPU implementation of per-step decay "
                              "(only its never-launched Triton kernel describes it)"}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, mode, budget_s=args.cpu_seconds)

    launch_mode = "CUDA graph replay" if graph is not None else "eager"
    if graph is not None:
        del graph           # holds NCCL calls at N > 1: released before the process group
    return {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms / steps, 5), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "bf16" if w.dtype == torch.bfloat16 else "f16",
        "data": DATA,
        "config": config_dict(w, world, strong, sem_label, args),
        "shard": {"pieces": [[p.s0, p.s1, p.c0, p.c1] for p in sc.pieces], "split_streams": sc.split,
                  "token_heads_rank0": rank_token_heads},
        "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e, "check": check,
        "gpu_launches": launches, "launch_mode": launch_mode,
        "clocks": clk.summary(),
    }


def config_dict(w, world, strong, sem_label, args):
    return dict(w.describe(), global_batch=w.B if strong else w.B * world, seq_len=w.T,
                semantics=sem_label,
                parallelism=((f"one problem sharded over {world} rank(s) by whole (batch,head) streams; "
                              "no data-path collective" if args.balance == "streams" else
                              f"one problem sharded over {world} rank(s) by (stream, chunk) ranges; "
                              "time-split streams exchange one carried state per direction")
                             if strong else f"(batch,head) weak scaling, {world} rank(s), no data-path collective"),
                l2="inputs larger than L2 (no flush needed)")


def run_check(args, w, sc, x, inp, decay, mode, need_dd, rank, world, dev):
    """Gather every rank's results on rank 0 and compare them with one GPU's run of
    the whole problem: normwise max|x - ref| / max|ref| per tensor, within 1e-3
    for the fp32 final state and 2e-2 for y and every gradient."""
    from simpletrain_b200.sharding import ShardedScan, cuda_scan_fns

    B, H, T, D = w.B, w.H, w.T, w.D
    need_ds0 = inp["s0"] is not None
    f32 = torch.float32
    shapes = {"y": ((B, H, T, D), w.dtype), "final_state": ((B, H, D, D), f32)}
    if w.backward:
        shapes.update({n: ((B, H, T, D), w.dtype) for n in ("dq", "dk", "dv", "dg")})
        if need_dd:
            shapes["ddecay"] = ((B, H, D), f32)
        if need_ds0:
            shapes["ds0"] = ((B, H, D, D), f32)

    def run(scan, xs):
        with torch.inference_mode():
            outs = scan.forward(xs)
            if w.backward:
                grads = scan.backward(xs, need_dd, need_ds0)
                outs = [dict(o, **g) for o, g in zip(outs, grads)]
            return outs

    def assemble(scan, outs):
        return scan.assemble(outs, shapes, dev)

    res = assemble(sc, run(sc, x))
    if rank != 0:
        return None
    one = ShardedScan(B, H, T, D, w.chunk, 1, 0, *cuda_scan_fns(w.chunk, mode))
    xo = one.load({"q": inp["q"], "k": inp["k"], "v": inp["v"], "g": inp["g"], "dy": inp["dy"],
                   "decay": decay, "s0": inp["s0"]})
    ref = assemble(one, run(one, xo))
    errs = {}
    for n in shapes:
        a, b = res[n].double(), ref[n].double()
        den = b.abs().max().item()
        errs[n] = (a - b).abs().max().item() / den if den > 0 else float((a - b).abs().max().item())
    tol = {n: (1e-3 if n == "final_state" else 2e-2) for n in errs}
    return {"against": "one GPU running the whole problem (same kernels, same inputs)",
            "max_rel": {n: float(f"{e:.3e}") for n, e in errs.items()},
            "ok": all(errs[n] <= tol[n] for n in errs)}


def run_e2e(args, w, sc, x, rank, world, dev, need_dd, need_ds0, tokens_per_step):
    """The same metric through the host-buffer API (``ShardedHostScan``): every
    step copies this rank's pieces (q, k, v, g, dy, decay, initial state) from
    pinned host memory to the device and every result back, inside the timed
    region; consecutive steps are pipelined so the two copy directions overlap
    each other and the kernels.  Then the copy floor: the same bytes moved by
    all ranks at once with nothing else running."""
    import torch.distributed as dist

    from simpletrain_b200.host_stream import ShardedHostScan

    def pinned(t):
        if not torch.is_tensor(t):
            return t
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h

    host = [{n: pinned(t) for n, t in p.items()} for p in x]
    runner = ShardedHostScan(sc, dev, need_dd, need_ds0, sets=3)
    h2d = ShardedHostScan.nbytes(host)
    steps = args.e2e_steps

    def run(n):
        # two steps in flight: step i is submitted before step i-2's results are read (the
        # submission itself waits for them before it queues its copies out)
        pend = []
        out = None
        for i in range(n + 2):
            if i < n:
                pend.append(runner.submit(host))
            if i >= 2:
                out = pend[i - 2].wait()
        return out

    out = run(3)          # every buffer set allocated (pinned host memory) before timing
    d2h = ShardedHostScan.nbytes(out)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    run(steps)
    b.record(stream)     # after the last step's results were awaited on the host
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    floor_ms = copy_floor(h2d, d2h, dev, world)
    t = torch.tensor([ms, floor_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, floor_ms = (float(v) for v in t.tolist())
    return {"value": round(tokens_per_step * steps / (ms / 1e3), 1), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "ms_per_step": round(ms / steps, 4),
            "copy_floor_ms_per_step": round(floor_ms, 4),
            "frac_of_copy_floor": round(floor_ms / (ms / steps), 4),
            "copy_floor": "each rank's h2d and d2h bytes moved at once (two streams, pinned memory) by all "
                          "ranks together, max over ranks",
            "api": "simpletrain_b200.host_stream.ShardedHostScan.submit + wait (pinned host pieces; copy-in / "
                   "scan / copy-out streams; three buffer sets, each step submitted before step i-2's "
                   "results are awaited)"}


def copy_floor(h2d, d2h, dev, world, reps=5):
    """Time moving h2d bytes host->device and d2h bytes device->host at once, on
    every rank together: the link's floor under this run's conditions."""
    import torch.distributed as dist
    hi = torch.empty(h2d, dtype=torch.uint8, pin_memory=True)
    di = torch.empty(h2d, dtype=torch.uint8, device=dev)
    do = torch.empty(d2h, dtype=torch.uint8, device=dev)
    ho = torch.empty(d2h, dtype=torch.uint8, pin_memory=True)
    s1, s2 = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    best = None
    for _ in range(reps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(dev)
        a.record(cur)
        s1.wait_stream(cur)
        s2.wait_stream(cur)
        with torch.cuda.stream(s1):
            di.copy_(hi, non_blocking=True)
        with torch.cuda.stream(s2):
            ho.copy_(do, non_blocking=True)
        cur.wait_stream(s1)
        cur.wait_stream(s2)
        b.record(cur)
        torch.cuda.synchronize()
        t = a.elapsed_time(b)
        best = t if best is None else min(best, t)
    return best


# --------------------------------------------------------------------------- #
# CPU legs (oracle port of the reference's torch path)
# --------------------------------------------------------------------------- #
def _cpu_sample_fn(w, mode, n_heads, T):
    """fwd(+bwd) of the oracle on n_heads (b, h) units of length T, in the
    workload's semantics (literal K V^T with a float decay at D == chunk)."""
    from oracle.kda_oracle import chunk_scan
    from simpletrain_b200.workloads import custom

    ws = custom(1, n_heads, T, w.D, dtype=w.dtype, backward=w.backward,
                decay_mean=w.decay_mean, s0_std=w.s0_std)
    inp = make_inputs(ws, seed=0)
    literal = mode == 1

    def run():
        leaves = [inp[n].float().requires_grad_(w.backward) for n in ("q", "k", "v", "g")]
        if literal:
            dl = float(inp["decay"].mean())
            wrt = leaves
            dec = dl
        else:
            dl = inp["decay"].float().requires_grad_(w.backward)
            wrt = leaves + [dl]
            dec = dl.view(1, n_heads, w.D, 1)
        y, S = chunk_scan(*leaves, dec, w.chunk, initial_state=inp["s0"],
                          mode="literal" if literal else "corrected")
        if w.backward:
            torch.autograd.grad([y], wrt, [inp["dy"].float()])
    return run


def cpu_baseline(w, mode, budget_s=15.0):
    """Time the oracle (a port of kernels/kda_kernel.py:244-297) on the host cores."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    heads, T = 1, w.T
    fn = _cpu_sample_fn(w, mode, heads, T)
    fn()
    t0 = time.perf_counter()
    fn()
    per = time.perf_counter() - t0
    heads = int(max(1, min(w.B * w.H, (budget_s / 4) / max(per, 1e-6))))
    fn = _cpu_sample_fn(w, mode, heads, T)
    fn()
    reps = 0
    t0 = time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    per = el / reps
    token_heads_per_s = heads * T / per
    return {"value": round(token_heads_per_s / w.H, 1), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{heads} (batch,head) unit(s) x T={T}, D={w.D}, "
                      f"{'fwd+bwd (autograd)' if w.backward else 'fwd'}, fp32, {reps} reps; "
                      f"tokens/s = token-heads/s / H", "seconds": round(el, 2)}


def run_reference(args, w, rank, world):
    if rank != 0:
        return None
    mode, _, _, sem_label = semantics(args, w)
    steps = args.steps if args.steps is not None else 10
    budget = 150.0
    step_budget = budget / max(1, steps + args.warmup)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    heads, T = 1, w.T
    fn = _cpu_sample_fn(w, mode, heads, T)
    fn()
    t0 = time.perf_counter()
    fn()
    per = time.perf_counter() - t0
    while per > step_budget and T > w.chunk:
        T = max(w.chunk, (T // 2) // w.chunk * w.chunk)
        fn = _cpu_sample_fn(w, mode, heads, T)
        fn()
        t0 = time.perf_counter()
        fn()
        per = time.perf_counter() - t0
    if per * 2 < step_budget:
        heads = int(max(1, min(w.B * w.H, step_budget / max(per, 1e-6) * 0.8)))
        fn = _cpu_sample_fn(w, mode, heads, T)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    el = time.perf_counter() - t0
    value = heads * T * steps / el / w.H
    sample = (f"{heads} (batch,head) unit(s) x T={T}, D={w.D} per step, "
              f"{'fwd+bwd (autograd)' if w.backward else 'fwd'}, fp32 oracle port of "
              f"kernels/kda_kernel.py:244-297 ({'literal K V^T' if mode == 1 else 'K^T V'} update); "
              "tokens/s = token-heads/s / H")
    strong = args.scaling == "strong"
    return {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(el / steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": config_dict(w, world, strong, sem_label, args),
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_layer(args):
    """The KDA layer forward + backward at the 1b shape (d_model 2560, 10 heads of
    128, B=16, T=2048, bf16), structured as SimpleTrain's layer (four projection
    GEMMs, the mean decay read back with .item()) and fused (one projection GEMM,
    decay on the device, free transpose): one JSON line each, CUDA-event time."""
    from simpletrain_b200.kda_layer import KDALayer, fused_forward, unfused_forward

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    B, T, Dm, H, Dh = 16, 2048, 2560, 10, 128
    layer = KDALayer(Dm, H, Dh).to(dev).to(torch.bfloat16)
    with torch.no_grad():
        layer.g_proj.weight.normal_(0.0, Dm ** -0.5)
    x = torch.randn(B, T, Dm, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    dy = torch.randn(B, T, Dm, device=dev, dtype=torch.bfloat16)
    for name, fwd, syncs in (("layer-structure (4 GEMMs, .item())", unfused_forward, 1),
                             ("fused (1 GEMM, no host sync)", fused_forward, 0)):
        def step():
            y = fwd(layer, x)
            y.backward(dy)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        n = args.steps or 20
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            step()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / n
        print(json.dumps({"layer": name, "ms_per_step": round(ms, 4), "tokens_per_s": round(B * T / (ms / 1e3), 1),
                          "host_syncs_per_step": syncs, "pass": "fwd+bwd",
                          "shape": {"B": B, "T": T, "d_model": Dm, "H": H, "D_head": Dh}}), flush=True)


def run_fused_ops(args):
    """One JSON line per fused op (fwd and bwd): HBM GB/s against the measured peak.

    Shapes are the 1b model's: tokens N = 16 x 2048, d_model 2560, FFN hidden
    6912, vocabulary 32000; bf16.  Algorithmic bytes = every operand read and
    written once.  Inputs exceed L2.
    """
    import simpletrain_b200.fused_ops  # noqa: F401  (loads the ops)
    peak = load_peaks()["hbm_gbs"]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(0)
    N, Dm, Hf, V = 16 * 2048, 2560, 6912, 32000
    bf = torch.bfloat16

    def mk(*shape):
        return torch.randn(*shape, generator=g).to(bf).to(dev)

    def timed(fn, n=50):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    ops = torch.ops.st_b200
    a, bb, dout = mk(N, Hf), mk(N, Hf), mk(N, Hf)
    x, r, dy, w = mk(N, Dm), mk(N, Dm), mk(N, Dm), mk(Dm)
    _, rstd = ops.rmsnorm_residual(x, r, w, 1e-6)
    logits = mk(N // 2, V)
    labels = torch.randint(0, V, (N // 2,), generator=g).to(dev)
    _, lse, _ = ops.cross_entropy(logits, labels, False)
    dl = torch.full((N // 2,), 1.0 / (N // 2), device=dev)
    e = 2  # bytes per bf16 element
    cases = [
        ("silu_mul fwd", lambda: ops.silu_mul(a, bb), 3 * N * Hf * e),
        ("silu_mul bwd", lambda: ops.silu_mul_bwd(a, bb, dout), 5 * N * Hf * e),
        ("rmsnorm_residual fwd", lambda: ops.rmsnorm_residual(x, r, w, 1e-6), 3 * N * Dm * e),
        ("rmsnorm_residual bwd", lambda: ops.rmsnorm_residual_bwd(x, w, rstd, dy), 3 * N * Dm * e),
        ("cross_entropy fwd (loss only)", lambda: ops.cross_entropy(logits, labels, False), (N // 2) * V * e),
        ("cross_entropy fwd (+softmax)", lambda: ops.cross_entropy(logits, labels, True), 2 * (N // 2) * V * e),
        ("cross_entropy bwd", lambda: ops.cross_entropy_bwd(logits, labels, lse, dl), 2 * (N // 2) * V * e),
    ]
    for name, fn, nbytes in cases:
        ms = timed(fn)
        gbs = nbytes / ms / 1e6
        print(json.dumps({"op": name, "ms": round(ms, 4), "GB_s": round(gbs, 1), "peak_GB_s": peak,
                          "frac": round(gbs / peak, 4), "algorithmic_bytes": nbytes,
                          "shape": {"tokens": N, "d_model": Dm, "ffn_hidden": Hf, "vocab": V}}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: ~3 s worth)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="1b-fwdbwd", choices=sorted(WORKLOADS))
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: one problem sharded over the ranks (default); weak: a full batch per rank")
    ap.add_argument("--balance", choices=["streams", "chunks"], default="streams",
                    help="strong scaling: whole streams per rank (default), or exactly balanced chunk ranges "
                         "with streams split in time between ranks")
    ap.add_argument("--shape", default=None,
                    help="B,H,T,D: run a custom shape (profiling / sweeps) instead of --workload")
    ap.add_argument("--fwd-only", action="store_true", help="with --shape: forward pass only")
    ap.add_argument("--per-step", action="store_true",
                    help="per-token decay semantics (one decay per head) instead of chunk-constant decay")
    ap.add_argument("--corrected", action="store_true",
                    help="at D == chunk, the K^T V update instead of the reference's literal one")
    ap.add_argument("--eager", action="store_true", help="launch each step eagerly instead of replaying a graph")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--fused-ops", action="store_true",
                    help="measure the fused silu*mul / RMSNorm / cross-entropy ops instead (one line each)")
    ap.add_argument("--layer", action="store_true",
                    help="measure the KDA layer fwd+bwd, structured as SimpleTrain's and fused (one line each)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.fused_ops:
        run_fused_ops(args)
        return
    if args.layer:
        run_layer(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = WORKLOADS[args.workload]
    if args.shape:
        from simpletrain_b200.workloads import custom
        B, H, T, D = (int(x) for x in args.shape.split(","))
        w = custom(B, H, T, D, backward=not args.fwd_only)

    if args.impl == "reference":
        out = run_reference(args, w, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        out = run_ours(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
