"""The sm_100a path against outputs of SimpleTrain's own code.

Fixtures (``tests/golden/make_golden.py``):

* ``cor_d128_*.pt`` -- the reference's ``_kda_chunked_scan_torch``
  (``kernels/kda_kernel.py:244-297``) with only its state-update einsum (``:294``)
  changed to the ``K^T V`` contraction: the semantics every D=128 model runs
  here (the shipped function raises at D=128).
* ``layer_*.pt`` -- SimpleTrain's ``KimiDeltaAttention`` (``models/kimi_k3.py:61-128``)
  itself, fp32 on the CPU, on seeded parameters and input: 100m variant (D=64,
  the shipped scan) and 1b variant (D=128, the one-line K^T V scan).  Here the
  same parameters run through ``kda_layer.KDALayer`` with the layer's own
  structure (``unfused_forward``) and the fused projection (``fused_forward``),
  the scan served by the drop-in.

Tolerance: normwise max|x - ref| / max|ref| <= 2e-2 for every output and
gradient (bf16 arithmetic against the reference's fp32).
"""
import os

import pytest
import torch

from oracle.kda_oracle import chunk_scan, max_rel
from simpletrain_b200 import device_status, kda_chunk, kda_chunked_scan
from simpletrain_b200.workloads import WORKLOADS, layer_input, layer_params, make_inputs, sketch_vectors

pytestmark = pytest.mark.gpu

TOL = 2e-2
DEV = "cuda"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert device_status() == 0, "a device-side bounded wait expired"


def _load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


def _check(pairs):
    errs = {n: max_rel(got.float().cpu(), ref.float()) for n, got, ref in pairs}
    bad = {n: e for n, e in errs.items() if not e <= TOL}
    assert not bad, f"max_rel above {TOL}: {bad} (all: {errs})"
    return errs


def _scan_with_grads(fn, f, cast=None):
    cast = cast or (lambda t: t)
    leaves = {n: cast(f[n].to(DEV)).detach().requires_grad_(True) for n in ("q", "k", "v", "g")}
    dec = f["decay"]
    if torch.is_tensor(dec):
        dec = dec.to(DEV).requires_grad_(True)
    y = fn(leaves["q"], leaves["k"], leaves["v"], leaves["g"], dec)
    (y.float() * f["dy"].to(DEV).float()).sum().backward()
    out = [("y", y, f["y"])] + [(f"d{n}", leaves[n].grad, f[f"d{n}"]) for n in ("q", "k", "v", "g")]
    if torch.is_tensor(dec):
        out.append(("ddecay", dec.grad, f["ddecay"]))
    return y, out


# --------------------------------------------------------------------------- #
# D = 128: the reference's function with the K^T V update
# --------------------------------------------------------------------------- #
def test_kda_chunk_matches_reference_kt_v_bf16(golden_dir):
    f = _load(golden_dir, "cor_d128_bf16.pt")
    _, pairs = _scan_with_grads(lambda q, k, v, g, d: kda_chunk(
        q, k, v, g, d.view(1, *d.shape[1:3]), None, f["chunk"], output_final_state=False)[0], f)
    _check(pairs)


def test_dropin_matches_reference_kt_v_bf16(golden_dir):
    """Through SimpleTrain's dispatch name with the default semantics ("auto":
    K^T V at D=128) and the reference's [1, H, D, 1] tensor decay."""
    f = _load(golden_dir, "cor_d128_bf16.pt")
    y, pairs = _scan_with_grads(lambda q, k, v, g, d: kda_chunked_scan(
        q, k, v, gate=g, decay=d, chunk_size=f["chunk"]), f)
    assert y.dtype == torch.bfloat16 and y.shape == f["y"].shape
    _check(pairs)


def test_dropin_fp32_without_triton_matches_reference_kt_v(golden_dir):
    """fp32 tensors with use_triton=False (the reference runs its fp32 torch loop
    there): y comes back in fp32 and gradients reach the fp32 leaves."""
    f = _load(golden_dir, "cor_d128_f32.pt")
    y, pairs = _scan_with_grads(lambda q, k, v, g, d: kda_chunked_scan(
        q, k, v, gate=g, decay=d, chunk_size=f["chunk"], use_triton=False), f)
    assert y.dtype == torch.float32
    for n, got, _ in pairs:
        assert got.dtype == torch.float32, n
    _check(pairs)


def test_dropin_fp32_without_triton_matches_reference_literal(golden_dir):
    f = _load(golden_dir, "lit_f32.pt")
    y, pairs = _scan_with_grads(lambda q, k, v, g, d: kda_chunked_scan(
        q, k, v, gate=g, decay=d, chunk_size=f["chunk"], use_triton=False), f)
    assert y.dtype == torch.float32
    _check(pairs)


def test_dropin_fp32_with_triton_asserts_like_reference():
    q = torch.randn(1, 1, 64, 64, device=DEV)
    with pytest.raises(AssertionError):
        kda_chunked_scan(q, q, q, use_triton=True)


# --------------------------------------------------------------------------- #
# SimpleTrain's KDA layer
# --------------------------------------------------------------------------- #
def _layer(f, dtype, use_triton=True):
    from simpletrain_b200.kda_layer import KDALayer
    layer = KDALayer(f["d_model"], f["n_heads"], f["d_head"], f["chunk"], dtype=dtype,
                     use_triton=use_triton)
    layer.load_state_dict(layer_params(f["d_model"], f["n_heads"], f["d_head"], f["seed_params"]))
    return layer.to(DEV).to(dtype)


def _layer_pairs(f, layer, forward, dtype):
    x, dy = layer_input(f["B"], f["T"], f["d_model"], f["seed_x"])
    x = x.to(DEV, dtype).requires_grad_(True)
    y = forward(layer, x)
    assert y.dtype == dtype and y.shape == f["y"].shape
    y.backward(dy.to(DEV, dtype))
    pairs = [("y", y.detach(), f["y"]), ("dx", x.grad, f["dx"]),
             ("dlog_decay", layer.log_decay.grad, f["dlog_decay"])]
    params = dict(layer.named_parameters())
    for pname, sk in f["grad_sketches"].items():
        gd = params[pname].grad.double().cpu()
        r_out, r_in = sketch_vectors(gd.shape[0], gd.shape[1], sk["seed"])
        pairs.append((f"{pname} W r", gd @ r_in, sk["W_r_in"]))
        pairs.append((f"{pname} r W", r_out @ gd, sk["r_out_W"]))
    return pairs


@pytest.mark.parametrize("name", ["layer_100m.pt", "layer_1b.pt"])
@pytest.mark.parametrize("structure", ["unfused", "fused"])
def test_simpletrain_layer_bf16_matches_reference_layer(golden_dir, name, structure):
    """The bf16 model (SimpleTrain's default dtype, config.py:65) against the
    reference layer's fp32 output and gradients."""
    from simpletrain_b200.kda_layer import fused_forward, unfused_forward
    f = _load(golden_dir, name)
    fwd = unfused_forward if structure == "unfused" else fused_forward
    _check(_layer_pairs(f, _layer(f, torch.bfloat16), fwd, torch.bfloat16))


@pytest.mark.parametrize("name", ["layer_100m.pt", "layer_1b.pt"])
def test_simpletrain_layer_fp32_without_triton_matches_reference_layer(golden_dir, name):
    """An fp32 model with use_triton=False (config.py:64-65), which the reference
    serves with its fp32 torch loop."""
    from simpletrain_b200.kda_layer import unfused_forward
    f = _load(golden_dir, name)
    _check(_layer_pairs(f, _layer(f, torch.float32, use_triton=False), unfused_forward, torch.float32))


# --------------------------------------------------------------------------- #
# the 100m workload in the semantics the reference computes there
# --------------------------------------------------------------------------- #
def test_config_100m_forward_through_dropin_literal():
    """B16 H8 T2048 D64 (128 streams: one work range per stream) through the
    drop-in with a float decay, as the 100m model calls it (models/kimi_k3.py:109-118):
    the reference's literal K V^T update, against the oracle in literal mode."""
    w = WORKLOADS["100m-fwd"]
    inp = make_inputs(w, seed=0)
    dscalar = float(inp["decay"].mean())
    q, k, v, g = (inp[n].to(DEV) for n in ("q", "k", "v", "g"))
    y = kda_chunked_scan(q, k, v, gate=g, decay=dscalar, chunk_size=w.chunk)
    ref, _ = chunk_scan(inp["q"].float(), inp["k"].float(), inp["v"].float(), inp["g"].float(),
                        dscalar, w.chunk, mode="literal")
    _check([("y", y, ref)])
    # and it is not the K^T V result: the two semantics differ at this size
    other, _ = chunk_scan(inp["q"][:1, :1].float(), inp["k"][:1, :1].float(), inp["v"][:1, :1].float(),
                          inp["g"][:1, :1].float(), dscalar, w.chunk, mode="corrected")
    assert max_rel(y[:1, :1].float().cpu(), other) > 10 * TOL
