"""Generate golden KDA vectors from SimpleTrain's own torch path.

Run in a checkout where the reference project is importable (it is not needed
anywhere else):

    python tests/golden/make_golden.py --reference /root/reference

Each fixture runs the reference function ``_kda_chunked_scan_torch``
(``kernels/kda_kernel.py:244-297``) unmodified -- its Triton path never
launches, so this function is what the reference computes on every device --
and stores inputs, outputs and autograd gradients.  The reference only runs
when D == chunk (its state update is ``K V^T``, ``:294``); the D=128 case
records the error it raises instead.

Fixtures (``tests/golden/*.pt``):
  lit_f32.pt        B1 H2 T128 D64, fp32, gate, float decay 0.93; y + grads q,k,v,g
  lit_bf16.pt       B1 H2 T192 D64, bf16, gate, tensor decay [1,H,D,1]; y + grads incl. decay
                    (three chunks, so the decay reaches the output through the state)
  lit_tail1.pt      B1 H1 T129 D64, fp32, no gate, float decay (1-token tail chunk)
  cpu_fwd_f32.pt    the seeded CPU workload (B2 H8 T512 D64 fp32, seed 0) with
                    decay = mean of the drawn per-channel decays: input checksums,
                    the first chunk of heads 0-1 and the last chunk
                    of heads 6-7 of y for batch 0, and per-chunk sums
  d128_error.pt     the message the reference raises at D=128, chunk 64
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from simpletrain_b200.workloads import WORKLOADS, make_inputs  # noqa: E402


def _inputs(B, H, T, D, dtype, seed, gate=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g)
    q = q / q.norm(dim=-1, keepdim=True)
    k = torch.randn(B, T, H, D, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, T, H, D, generator=g)
    gt = torch.sigmoid(torch.randn(B, T, H, D, generator=g)) if gate else None
    dy = torch.randn(B, T, H, D, generator=g)
    cv = lambda x: None if x is None else x.to(dtype).transpose(1, 2).contiguous()
    return cv(q), cv(k), cv(v), cv(gt), cv(dy)


def _run(fn, q, k, v, gt, dy, decay, C):
    leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]
    gl = gt.detach().clone().requires_grad_(True) if gt is not None else None
    dl = decay.detach().clone().requires_grad_(True) if torch.is_tensor(decay) else decay
    y = fn(*leaves, gl, dl, C)
    (y.float() * dy.float()).sum().backward()
    out = {"y": y.detach(), "dq": leaves[0].grad, "dk": leaves[1].grad, "dv": leaves[2].grad}
    if gl is not None:
        out["dg"] = gl.grad
    if torch.is_tensor(dl):
        out["ddecay"] = dl.grad
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from kernels.kda_kernel import _kda_chunked_scan_torch as ref  # noqa: E402

    torch.manual_seed(0)
    # 1) literal fp32 with gate and float decay
    q, k, v, gt, dy = _inputs(1, 2, 128, 64, torch.float32, 11)
    res = _run(ref, q, k, v, gt, dy, 0.93, 64)
    torch.save({"q": q, "k": k, "v": v, "g": gt, "dy": dy, "decay": 0.93, "chunk": 64, **res},
               os.path.join(HERE, "lit_f32.pt"))

    # 2) literal bf16 with tensor decay [1,H,D,1] (autograd gives its gradient)
    q, k, v, gt, dy = _inputs(1, 2, 192, 64, torch.bfloat16, 12)
    decay = torch.sigmoid(torch.randn(1, 2, 64, 1, generator=torch.Generator().manual_seed(13)) + 3.0)
    res = _run(ref, q, k, v, gt, dy, decay, 64)
    torch.save({"q": q, "k": k, "v": v, "g": gt, "dy": dy, "decay": decay, "chunk": 64, **res},
               os.path.join(HERE, "lit_bf16.pt"))

    # 3) literal, no gate, T % 64 == 1 (the [1,1] tail update broadcasts)
    q, k, v, _, dy = _inputs(1, 1, 129, 64, torch.float32, 14, gate=False)
    y = ref(q, k, v, None, 0.9, 64)
    torch.save({"q": q, "k": k, "v": v, "decay": 0.9, "chunk": 64, "y": y},
               os.path.join(HERE, "lit_tail1.pt"))

    # 4) the seeded CPU workload through the unmodified reference
    w = WORKLOADS["cpu-fwd-f32"]
    inp = make_inputs(w, seed=0)
    dscalar = float(inp["decay"].mean())
    y = ref(inp["q"], inp["k"], inp["v"], inp["g"], dscalar, w.chunk)
    sums = {n: inp[n].double().sum().item() for n in ("q", "k", "v", "g", "decay")}
    yc = y.double().reshape(w.B, w.H, w.T // w.chunk, w.chunk, w.D)
    torch.save({
        "workload": w.name, "seed": 0, "decay_scalar": dscalar, "input_sums": sums,
        "y_first": y[0, :2, :w.chunk].clone(), "y_last": y[0, -2:, -w.chunk:].clone(),
        "chunk_sum": yc.sum(dim=(3, 4)), "chunk_sumsq": (yc * yc).sum(dim=(3, 4)),
    }, os.path.join(HERE, "cpu_fwd_f32.pt"))

    # 5) the D=128 failure
    q, k, v, gt, _ = _inputs(1, 1, 128, 128, torch.float32, 15)
    try:
        ref(q, k, v, gt, 0.9, 64)
        msg = ""
    except RuntimeError as e:
        msg = str(e)
    torch.save({"message": msg}, os.path.join(HERE, "d128_error.pt"))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
