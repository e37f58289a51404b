"""Generate golden KDA vectors from SimpleTrain's own torch code.

Run in a checkout where the reference project is importable (it is not needed
anywhere else); its location is required, as an argument or in the
environment variable SIMPLETRAIN_REFERENCE:

    python tests/golden/make_golden.py --reference <path to SimpleTrain>

The reference's Triton path never launches, so its torch function
``_kda_chunked_scan_torch`` (``kernels/kda_kernel.py:244-297``) is what it
computes on every device.  Two forms of that function are run here:

* as shipped (the "literal" state update ``K V^T``, ``:294``), which only runs
  when D == chunk;
* for D = 128, where the shipped function raises, the function's own source
  with exactly one line changed: the state-update einsum at ``:294`` becomes
  the ``K^T V`` contraction (``"bhpd,bhpe->bhde"``).  ``corrected_reference``
  checks that the two sources differ in that single line before it executes
  the changed one, so these fixtures are the reference's code, not a
  restatement of it.

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
  cor_d128_f32.pt   D=128 through the one-line K^T V form: B1 H1 T136 (two chunks and
                    an 8-token tail), fp32, gate, float decay 0.95; y + grads q,k,v,g
  cor_d128_bf16.pt  the same form on two heads of the 1b workload's distributions
                    (q, k L2-normalised, per-channel decay sigmoid(N(3,1)) as a
                    [1,H,D,1] tensor): B1 H2 T200 (three chunks and an 8-token
                    tail), bf16; y + grads q,k,v,g,decay
  layer_100m.pt     SimpleTrain's own KimiDeltaAttention (models/kimi_k3.py:61-128),
                    100m variant (d_model 512, 8 heads of 64), fp32 on the CPU,
                    use_triton=False, seeded parameters (workloads.layer_params) and
                    input (workloads.layer_input), B1 T192: the layer output y, dL/dx,
                    dL/dlog_decay and sketches (W r_in, r_out W) of every weight
                    gradient, for L = sum(y * dy)
  layer_1b.pt       the same for the 1b variant (d_model 1280, 10 heads of 128),
                    B1 T136, with the one-line K^T V form in place of the
                    reference's scan (which raises at D=128)
"""
from __future__ import annotations

import argparse
import difflib
import inspect
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from simpletrain_b200.workloads import (WORKLOADS, layer_input, layer_params,  # noqa: E402
                                        make_inputs, sketch_vectors)

# the reference's state-update contraction (kernels/kda_kernel.py:294) and its K^T V form
LITERAL_KV = 'torch.einsum("bhpd,bhqd->bhpq", kc, vc)'
CORRECTED_KV = 'torch.einsum("bhpd,bhpe->bhde", kc, vc)'

LAYER_SKETCH_SEED = 7


def corrected_reference(kk):
    """``kk._kda_chunked_scan_torch`` with only the ``:294`` einsum changed to K^T V.

    Reads the function's source from the reference module, replaces the one
    contraction, asserts that exactly one source line differs (and that it is
    the state update), and executes the result in a copy of the module's
    namespace.
    """
    src = inspect.getsource(kk._kda_chunked_scan_torch)
    if src.count(LITERAL_KV) != 1:
        raise SystemExit(f"expected the state-update einsum {LITERAL_KV!r} exactly once")
    new = src.replace(LITERAL_KV, CORRECTED_KV)
    a, b = src.splitlines(), new.splitlines()
    diff = [ln for ln in difflib.unified_diff(a, b, lineterm="", n=0)
            if ln[:1] in "+-" and not ln.startswith(("+++", "---"))]
    assert len(a) == len(b) and len(diff) == 2, diff
    assert diff[0].lstrip("-").strip().startswith("full_kv = " + LITERAL_KV), diff
    assert diff[1].lstrip("+").strip().startswith("full_kv = " + CORRECTED_KV), diff
    ns = dict(vars(kk))
    code = compile(new, f"{kk.__file__} (_kda_chunked_scan_torch with K^T V at :294)", "exec")
    exec(code, ns)  # noqa: S102 -- the reference's own function, one einsum changed
    return ns["_kda_chunked_scan_torch"]


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


def _layer_fixture(variant, T, seed_params, seed_x):
    """Run SimpleTrain's KimiDeltaAttention (fp32, CPU, use_triton=False) on seeded
    parameters and input; return its output, input gradient and gradient sketches."""
    from config import get_config
    from models.kimi_k3 import KimiDeltaAttention

    cfg = get_config(variant, dtype="float32", use_triton=False)
    layer = KimiDeltaAttention(cfg)
    layer.load_state_dict(layer_params(cfg.d_model, cfg.n_heads, cfg.d_head, seed_params))
    x, dy = layer_input(1, T, cfg.d_model, seed_x)
    x = x.requires_grad_(True)
    y = layer(x)
    (y * dy).sum().backward()
    sketches = {}
    for i, (name, p) in enumerate(sorted(layer.named_parameters())):
        if p.dim() != 2:
            continue
        r_out, r_in = sketch_vectors(p.shape[0], p.shape[1], LAYER_SKETCH_SEED + i)
        gd = p.grad.double()
        sketches[name] = {"W_r_in": gd @ r_in, "r_out_W": r_out @ gd, "seed": LAYER_SKETCH_SEED + i}
    return {
        "variant": variant, "d_model": cfg.d_model, "n_heads": cfg.n_heads, "d_head": cfg.d_head,
        "chunk": cfg.kda_chunk_size, "B": 1, "T": T, "seed_params": seed_params, "seed_x": seed_x,
        "y": y.detach(), "dx": x.grad.detach(), "dlog_decay": layer.log_decay.grad.detach(),
        "grad_sketches": sketches,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SIMPLETRAIN_REFERENCE"),
                    help="root of a SimpleTrain checkout (or set SIMPLETRAIN_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <SimpleTrain checkout> or set SIMPLETRAIN_REFERENCE")
    sys.path.insert(0, os.path.abspath(args.reference))
    import kernels.kda_kernel as kk  # noqa: E402
    ref = kk._kda_chunked_scan_torch
    ref_kt_v = corrected_reference(kk)

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

    # 6) D=128 through the reference's function with the K^T V update, fp32, float decay
    q, k, v, gt, dy = _inputs(1, 1, 136, 128, torch.float32, 16)
    res = _run(ref_kt_v, q, k, v, gt, dy, 0.95, 64)
    torch.save({"q": q, "k": k, "v": v, "g": gt, "dy": dy, "decay": 0.95, "chunk": 64, **res},
               os.path.join(HERE, "cor_d128_f32.pt"))

    # 7) the same in bf16 on two heads of the 1b workload (per-channel tensor decay)
    q, k, v, gt, dy = _inputs(1, 2, 200, 128, torch.bfloat16, 17)
    decay = torch.sigmoid(torch.randn(1, 2, 128, 1, generator=torch.Generator().manual_seed(18)) + 3.0)
    res = _run(ref_kt_v, q, k, v, gt, dy, decay, 64)
    torch.save({"q": q, "k": k, "v": v, "g": gt, "dy": dy, "decay": decay, "chunk": 64, **res},
               os.path.join(HERE, "cor_d128_bf16.pt"))

    # 8) SimpleTrain's KDA layer, 100m variant (D = chunk: the shipped scan)
    torch.save(_layer_fixture("100m", 192, 0, 1), os.path.join(HERE, "layer_100m.pt"))

    # 9) the 1b variant, with the K^T V scan in place of the one that raises
    kk._kda_chunked_scan_torch = ref_kt_v
    try:
        torch.save(_layer_fixture("1b", 136, 2, 3), os.path.join(HERE, "layer_1b.pt"))
    finally:
        kk._kda_chunked_scan_torch = ref
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
