#!/usr/bin/env python
"""KDA chunked-scan throughput on B200: forward + backward tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload 1b-fwdbwd]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)
    python bench.py --impl reference ...                     (CPU arm)

One step = one forward + backward pass of the KDA scan over one batch of the
workload (default: the 1b-variant shape B=16, H=10, T=2048, D=128, chunk 64,
bf16).  Work shards by (batch, head): every rank runs its own full batch of
independent (b, h) units with no collective on the data path (weak scaling);
``value`` = tokens all ranks processed / max-over-ranks device time.

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


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


def algorithmic(w, rank_heads=None):
    """Algorithmic HBM bytes and flops per launch-group (per rank, per step).

    Per token-head with chunk C: forward reads q,k,v,g and writes y (10*D bytes
    in bf16) and costs 4CD + 4D^2 flops; backward reads q,k,v,g,dy and writes
    dq,dk,dv,dg (18*D bytes) and costs 8CD + 8D^2 flops.  Plus the fp32 DxD
    state once per (b, h) per direction.
    """
    B, H, T, D, C = w.B, w.H, w.T, w.D, w.chunk
    th = B * H * T
    bh = B * H
    esz = torch.finfo(w.dtype).bits // 8
    fwd_bytes = th * 5 * D * esz + bh * D * D * 4
    bwd_bytes = th * 9 * D * esz + bh * D * D * 4 + bh * D * 4
    return {
        "fwd": {"bytes": fwd_bytes, "flops": th * (4 * C * D + 4 * D * D)},
        "bwd": {"bytes": bwd_bytes, "flops": th * (8 * C * D + 8 * D * D)},
    }


# --------------------------------------------------------------------------- #
# clocks during the timed region
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
            # nvidia-smi takes a moment to start: wait (at most 3 s) for its first
            # sample so that even a short timed region is covered
            t0 = time.time()
            while os.path.getsize(self.path) == 0 and self.proc.poll() is None and time.time() - t0 < 3.0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
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
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


# --------------------------------------------------------------------------- #
# our arm
# --------------------------------------------------------------------------- #
def traffic_from_profiles(w, kernel: str):
    """DRAM bytes per launch-group from a committed ncu summary, scaled by units."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as fh:
        d = json.load(fh)
    ent = d.get(f"{kernel}:D{w.D}")
    if not ent:
        return None
    return ent["bytes_per_token_head"] * w.B * w.H * w.T


def run_ours(args, w, rank, world, local_rank):
    import torch.distributed as dist

    import simpletrain_b200.ops  # noqa: F401  (loads the ops)
    from simpletrain_b200 import _ffi
    from simpletrain_b200.ops import device_status, kda_chunk

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    inp = make_inputs(w, seed=rank, device=dev)
    q, k, v, g, dy, decay, s0 = (inp[n] for n in ("q", "k", "v", "g", "dy", "decay", "s0"))
    B, H, T, D = w.B, w.H, w.T, w.D
    if args.per_step:
        # per-token decay, one value per head (the first channel's)
        mode, need_dd = 2, False
        dec = decay[:, :1].expand(B, H, D)
    else:
        mode, need_dd = 0, True
        dec = decay.expand(B, H, D)
    fwd = torch.ops.kda_b200.chunk_fwd
    bwd = torch.ops.kda_b200.chunk_bwd

    # the ops are called directly (their backward explicitly): no autograd
    # bookkeeping, which would add a Python layer to every call
    inference = torch.inference_mode()
    inference.__enter__()

    def step():
        y, sT = fwd(q, k, v, g, dec, 0.0, s0, w.chunk, mode, True)
        if w.backward:
            return bwd(q, k, v, g, dy, dec, 0.0, s0, None, None, w.chunk, mode, need_dd, s0 is not None)
        return y

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    steps = args.steps
    if steps is None:
        t0 = time.perf_counter()
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        per = (time.perf_counter() - t0) / 3
        steps = int(min(5000, max(10, 3.0 / max(per, 1e-6))))
        if world > 1:
            t = torch.tensor([steps], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            steps = int(t.item())

    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _ffi.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        start.record(stream)
        for i in range(steps):
            e0, e1, e2 = ev[i]
            e0.record(stream)
            y, sT = fwd(q, k, v, g, dec, 0.0, s0, w.chunk, mode, True)
            e1.record(stream)
            if w.backward:
                bwd(q, k, v, g, dy, dec, 0.0, s0, None, None, w.chunk, mode, need_dd, s0 is not None)
            e2.record(stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    launches = _ffi.launch_count() - launches0
    ms = start.elapsed_time(end)
    fwd_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1, _ in ev)
    bwd_ms = statistics.mean(e1.elapsed_time(e2) for _, e1, e2 in ev) if w.backward else 0.0
    t = torch.tensor([ms, fwd_ms, bwd_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_ms, bwd_ms = (float(x) for x in t.tolist())
    inference.__exit__(None, None, None)
    status = device_status(dev)
    if status:
        raise RuntimeError(f"device-side KDA status {status}")

    tokens_per_step = world * B * T
    value = tokens_per_step * steps / (ms / 1e3)

    # ---- roofline of the dominant launch group ---------------------------------
    peaks = load_peaks()
    alg = algorithmic(w)
    groups = {"fwd": fwd_ms}
    if w.backward:
        groups["bwd"] = bwd_ms
    dom = max(groups, key=groups.get)
    achieved = alg[dom]["bytes"] / (groups[dom] / 1e3) / 1e9
    traffic = traffic_from_profiles(w, dom)
    kernels = {}
    for name, t_ms in groups.items():
        kernels[name] = {"ms": round(t_ms, 4),
                         "GB_s": round(alg[name]["bytes"] / (t_ms / 1e3) / 1e9, 1),
                         "TFLOP_s": round(alg[name]["flops"] / (t_ms / 1e3) / 1e12, 1)}
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": traffic, "kernel": f"kda_{dom}",
                "peak_source": peaks["source"],
                "tensor_frac": round(alg[dom]["flops"] / (groups[dom] / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
                "step_frac": round(sum(alg[n]["bytes"] for n in groups) / (ms / steps / 1e3) / 1e9
                                   / peaks["hbm_gbs"], 4)}

    # ---- end to end through the public API with host buffers --------------------
    e2e = run_e2e(args, w, rank, world, dev, inp) if not args.no_e2e else None

    # ---- CPU baseline (rank 0, N = 1) ----------------------------------------------
    cpu = None
    if args.per_step:
        cpu = {"unavailable": "the reference has no CPU implementation of per-step decay "
                              "(only its never-launched Triton kernel describes it)"}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, budget_s=args.cpu_seconds)

    return {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms / steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "f16",
        "data": "synthetic (seeded; q,k L2-normalised N(0,1), v N(0,1), g sigmoid(N(0,1)), "
                "per-channel decay sigmoid(N(3,1)))",
        "config": dict(w.describe(), global_batch=w.B * world, seq_len=w.T,
                       semantics="per-step decay (one per head)" if args.per_step else "chunk-constant decay",
                       parallelism=f"(batch,head) shards, {world} rank(s), no data-path collective",
                       l2="inputs larger than L2 (no flush needed)"),
        "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": launches, "clocks": clk.summary(),
    }


def run_e2e(args, w, rank, world, dev, inp):
    """Same metric through the public host-buffer API (``HostScan``): each step
    copies its inputs (q, k, v, g, dy, decay, initial state) from pinned host
    memory to the device and its results (y, final state, dq, dk, dv, dg,
    d_decay, d_initial_state) back, inside the timed region; the batch is
    pipelined in slices so both copy directions overlap the kernels, and each
    step is submitted before the previous step's results are awaited, so one
    step's copies in overlap the previous step's copies out."""
    import torch.distributed as dist

    from simpletrain_b200.host_stream import HostScan

    names = ["q", "k", "v", "g", "dy"] if w.backward else ["q", "k", "v", "g"]

    def pinned_like(t):
        return torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device="cpu", pin_memory=True)

    extra = ["decay"] + (["s0"] if inp["s0"] is not None else [])
    host = {n: pinned_like(inp[n]) for n in names + extra}
    for n in names + extra:
        host[n].copy_(inp[n])
    # per-step: one decay per head (the first channel's), not differentiated
    decay = host["decay"][:, 0].contiguous() if args.per_step else host["decay"]
    scan = HostScan(dev, slices=args.e2e_slices, chunk_size=w.chunk, per_step=args.per_step)
    steps = args.e2e_steps
    h2d = sum(host[n].numel() * host[n].element_size() for n in names + ["s0"] if n in host)
    h2d += decay.numel() * decay.element_size()
    d2h = 0

    def run(n):
        """n steps, each submitted before the previous one's results are awaited."""
        nonlocal d2h
        pend = None
        for i in range(n + 1):
            nxt = None
            if i < n:
                nxt = scan.submit(host["q"], host["k"], host["v"], host["g"], decay, dy=host.get("dy"),
                                  initial_state=host.get("s0"))
            if pend is not None:
                out = pend.wait()
                d2h = sum(o.numel() * o.element_size() for o in out.values())
            pend = nxt

    run(2)
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
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": round(world * w.B * w.T * steps / (ms / 1e3), 1), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "slices": scan.slices if scan.slices is not None else min(w.B, 16),
            "api": "simpletrain_b200.host_stream.HostScan.submit + wait (pinned host buffers, batch slices "
                   "pipelined over copy-in / scan / copy-out streams, each step submitted before the "
                   "previous step's results are awaited)"}


# --------------------------------------------------------------------------- #
# CPU legs (oracle port of the reference's torch path)
# --------------------------------------------------------------------------- #
def _cpu_sample_fn(w, n_heads, T):
    """fwd(+bwd) of the oracle on n_heads (b, h) units of length T."""
    from oracle.kda_oracle import chunk_scan
    from simpletrain_b200.workloads import custom

    sub = w
    ws = custom(1, n_heads, T, sub.D, dtype=sub.dtype, backward=sub.backward,
                decay_mean=sub.decay_mean, s0_std=sub.s0_std)
    inp = make_inputs(ws, seed=0)

    def run():
        leaves = [inp[n].float().requires_grad_(sub.backward) for n in ("q", "k", "v", "g")]
        dl = inp["decay"].float().requires_grad_(sub.backward)
        dec = dl.view(1, n_heads, sub.D, 1)
        y, S = chunk_scan(*leaves, dec, sub.chunk,
                          initial_state=inp["s0"], mode="corrected")
        if sub.backward:
            torch.autograd.grad([y], leaves + [dl], [inp["dy"].float()])
    return run


def cpu_baseline(w, budget_s=15.0, max_step_s=None):
    """Time the oracle (a port of kernels/kda_kernel.py:244-297) on the host cores."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    heads = 1
    T = w.T
    fn = _cpu_sample_fn(w, heads, T)
    fn()
    t0 = time.perf_counter()
    fn()
    per = time.perf_counter() - t0
    if max_step_s is not None:
        while per > max_step_s and T > w.chunk:
            T = max(w.chunk, (T // 2) // w.chunk * w.chunk)
            fn = _cpu_sample_fn(w, heads, T)
            fn()
            t0 = time.perf_counter()
            fn()
            per = time.perf_counter() - t0
    else:
        heads = int(max(1, min(w.B * w.H, (budget_s / 4) / max(per, 1e-6))))
        fn = _cpu_sample_fn(w, heads, T)
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
    steps = args.steps if args.steps is not None else 10
    budget = 150.0
    step_budget = budget / max(1, steps + args.warmup)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    heads, T = 1, w.T
    fn = _cpu_sample_fn(w, heads, T)
    fn()
    t0 = time.perf_counter()
    fn()
    per = time.perf_counter() - t0
    while per > step_budget and T > w.chunk:
        T = max(w.chunk, (T // 2) // w.chunk * w.chunk)
        fn = _cpu_sample_fn(w, heads, T)
        fn()
        t0 = time.perf_counter()
        fn()
        per = time.perf_counter() - t0
    if per * 2 < step_budget:
        heads = int(max(1, min(w.B * w.H, step_budget / max(per, 1e-6) * 0.8)))
        fn = _cpu_sample_fn(w, heads, T)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    el = time.perf_counter() - t0
    value = heads * T * steps / el / w.H
    sample = (f"{heads} (batch,head) unit(s) x T={T}, D={w.D} per step, "
              f"{'fwd+bwd (autograd)' if w.backward else 'fwd'}, fp32 oracle port of "
              f"kernels/kda_kernel.py:244-297 (K^T V update); tokens/s = token-heads/s / H")
    return {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(el / steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": dict(w.describe(), global_batch=w.B * world, seq_len=w.T),
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
    ap.add_argument("--shape", default=None,
                    help="B,H,T,D: run a custom shape (profiling / sweeps) instead of --workload")
    ap.add_argument("--fwd-only", action="store_true", help="with --shape: forward pass only")
    ap.add_argument("--per-step", action="store_true",
                    help="per-token decay semantics (one decay per head) instead of chunk-constant decay")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-slices", type=int, default=None,
                    help="batch slices of the host-buffer pipeline (default min(B, 16))")
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
