"""The oracle against the reference's own outputs and against known answers.

The golden vectors were produced by running SimpleTrain's unmodified
``_kda_chunked_scan_torch`` (``kernels/kda_kernel.py:244-297``); see
``tests/golden/make_golden.py``.  Errors are normwise: max|x-ref| / max|ref|.
"""
import os

import pytest
import torch

from oracle.kda_oracle import (chunk_scan, decay_bhd1, manual_backward, max_rel,
                               naive_recurrence)
from simpletrain_b200.workloads import WORKLOADS, custom, make_inputs


def _load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


def _grads(fn, q, k, v, g, decay, dy):
    leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]
    gl = g.detach().clone().requires_grad_(True) if g is not None else None
    dl = decay.detach().clone().requires_grad_(True) if torch.is_tensor(decay) else decay
    y = fn(*leaves, gl, dl)
    (y.float() * dy.float()).sum().backward()
    out = {"y": y.detach(), "dq": leaves[0].grad, "dk": leaves[1].grad, "dv": leaves[2].grad}
    if gl is not None:
        out["dg"] = gl.grad
    if torch.is_tensor(dl):
        out["ddecay"] = dl.grad
    return out


# --------------------------------------------------------------------------- #
# pinning against the reference
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("name,tol", [("lit_f32.pt", 1e-6), ("lit_bf16.pt", 1e-2)])
def test_literal_matches_reference_fixture(golden_dir, name, tol):
    f = _load(golden_dir, name)
    C = f["chunk"]
    res = _grads(lambda q, k, v, g, d: chunk_scan(q, k, v, g, d, C, mode="literal")[0],
                 f["q"], f["k"], f["v"], f["g"], f["decay"], f["dy"])
    for key in ("y", "dq", "dk", "dv", "dg") + (("ddecay",) if "ddecay" in f else ()):
        assert res[key].dtype == f[key].dtype, key
        assert max_rel(res[key], f[key]) <= tol, (key, max_rel(res[key], f[key]))


def test_literal_tail_of_one_token(golden_dir):
    f = _load(golden_dir, "lit_tail1.pt")
    y, _ = chunk_scan(f["q"], f["k"], f["v"], None, f["decay"], f["chunk"], mode="literal")
    assert max_rel(y, f["y"]) <= 1e-6


def test_seeded_cpu_workload_matches_reference(golden_dir):
    f = _load(golden_dir, "cpu_fwd_f32.pt")
    w = WORKLOADS[f["workload"]]
    inp = make_inputs(w, seed=f["seed"])
    for n, s in f["input_sums"].items():
        assert abs(inp[n].double().sum().item() - s) <= 1e-6 * max(1.0, abs(s)), \
            f"seeded generator drifted for {n}"
    y, _ = chunk_scan(inp["q"], inp["k"], inp["v"], inp["g"], f["decay_scalar"], w.chunk,
                      mode="literal")
    assert max_rel(y[0, :2, :w.chunk], f["y_first"]) <= 1e-6
    assert max_rel(y[0, -2:, -w.chunk:], f["y_last"]) <= 1e-6
    yc = y.double().reshape(w.B, w.H, w.T // w.chunk, w.chunk, w.D)
    assert max_rel(yc.sum(dim=(3, 4)), f["chunk_sum"]) <= 1e-5
    assert max_rel((yc * yc).sum(dim=(3, 4)), f["chunk_sumsq"]) <= 1e-5


@pytest.mark.parametrize("name,tol", [("cor_d128_f32.pt", 1e-5), ("cor_d128_bf16.pt", 1e-2)])
def test_corrected_matches_reference_kt_v_fixture(golden_dir, name, tol):
    """The corrected (K^T V) mode against the reference's own function with only
    its :294 einsum changed (D=128, ragged tail, float and per-channel decay)."""
    f = _load(golden_dir, name)
    C = f["chunk"]
    res = _grads(lambda q, k, v, g, d: chunk_scan(q, k, v, g, d, C, mode="corrected")[0],
                 f["q"], f["k"], f["v"], f["g"], f["decay"], f["dy"])
    assert f["q"].shape[-1] == 128 and f["q"].shape[2] % C != 0
    for key in ("y", "dq", "dk", "dv", "dg") + (("ddecay",) if "ddecay" in f else ()):
        assert res[key].dtype == f[key].dtype, key
        assert max_rel(res[key], f[key]) <= tol, (key, max_rel(res[key], f[key]))


def test_corrected_fixture_generator_changes_one_line():
    """The generator's one-line change, checked on a synthetic source: exactly the
    state-update einsum differs, so the D=128 fixtures run the reference's code."""
    import types

    from tests.golden.make_golden import CORRECTED_KV, LITERAL_KV, corrected_reference
    src = ("import torch\n"
           "def _kda_chunked_scan_torch(kc, vc):\n"
           "    s = 0\n"
           f"    full_kv = {LITERAL_KV}     # [B,H,D,D]\n"
           "    return full_kv\n")
    mod = types.ModuleType("fake_kda")
    mod.__file__ = "fake_kda.py"
    exec(compile(src, "fake_kda.py", "exec"), mod.__dict__)
    import inspect
    import linecache
    linecache.cache["fake_kda.py"] = (len(src), None, src.splitlines(True), "fake_kda.py")
    assert "bhpq" in inspect.getsource(mod._kda_chunked_scan_torch)
    fn = corrected_reference(mod)
    kc = torch.randn(1, 1, 5, 3)
    vc = torch.randn(1, 1, 5, 3)
    assert torch.allclose(fn(kc, vc), kc.transpose(-1, -2) @ vc)
    assert CORRECTED_KV != LITERAL_KV


@pytest.mark.parametrize("name,mode", [("layer_100m.pt", "literal"), ("layer_1b.pt", "corrected")])
def test_layer_fixture_matches_oracle_layer(golden_dir, name, mode):
    """SimpleTrain's KimiDeltaAttention output and gradients (fp32, CPU) against the
    oracle's restatement of the layer on the same seeded parameters and input."""
    from oracle.kda_oracle import layer_forward
    from simpletrain_b200.workloads import layer_input, layer_params, sketch_vectors
    f = _load(golden_dir, name)
    params = {n: p.requires_grad_(True) for n, p in
              layer_params(f["d_model"], f["n_heads"], f["d_head"], f["seed_params"]).items()}
    x, dy = layer_input(f["B"], f["T"], f["d_model"], f["seed_x"])
    x.requires_grad_(True)
    y = layer_forward(params, x, f["n_heads"], f["d_head"], f["chunk"], mode)
    (y * dy).sum().backward()
    assert max_rel(y, f["y"]) <= 1e-5
    assert max_rel(x.grad, f["dx"]) <= 1e-5
    assert max_rel(params["log_decay"].grad, f["dlog_decay"]) <= 1e-5
    for pname, sk in f["grad_sketches"].items():
        gd = params[pname].grad.double()
        r_out, r_in = sketch_vectors(gd.shape[0], gd.shape[1], sk["seed"])
        assert max_rel(gd @ r_in, sk["W_r_in"]) <= 1e-5, pname
        assert max_rel(r_out @ gd, sk["r_out_W"]) <= 1e-5, pname


def test_literal_fails_like_reference_at_d128(golden_dir):
    f = _load(golden_dir, "d128_error.pt")
    q = torch.randn(1, 1, 128, 128)
    with pytest.raises(RuntimeError) as e:
        chunk_scan(q, q, q, q, 0.9, 64, mode="literal")
    assert str(e.value) == f["message"]


# --------------------------------------------------------------------------- #
# known answers for the corrected form
# --------------------------------------------------------------------------- #
def _small(B=2, H=3, T=200, D=32, seed=0):
    g = torch.Generator().manual_seed(seed)
    mk = lambda: torch.randn(B, H, T, D, generator=g, dtype=torch.float64)
    return mk(), mk(), mk(), torch.sigmoid(mk())


def test_decay_one_is_full_causal_linear_attention():
    q, k, v, g = _small()
    T = q.shape[2]
    full = g * (torch.matmul(q, k.transpose(-1, -2)).tril() @ v)
    for C in (16, 64, 100):
        y, _ = chunk_scan(q, k, v, g, 1.0, C, compute_dtype=torch.float64)
        assert max_rel(y, full) < 1e-12, C
    assert T % 16 != 0 or True


def test_matches_per_token_restatement():
    q, k, v, g = _small(T=150)
    s0 = torch.randn(2, 3, 32, 32, dtype=torch.float64)
    y, S = chunk_scan(q, k, v, g, 0.9, 64, initial_state=s0, compute_dtype=torch.float64)
    yn, Sn = naive_recurrence(q, k, v, g, 0.9, 64, initial_state=s0)
    assert max_rel(y, yn) < 1e-12 and max_rel(S, Sn) < 1e-12


def test_split_at_chunk_boundary_with_state_handoff():
    q, k, v, g = _small(T=320)
    d = torch.rand(3, 32, dtype=torch.float64) * 0.2 + 0.8
    db = decay_bhd1(d, 2, 3, 32, dtype=torch.float64)
    y, S = chunk_scan(q, k, v, g, db, 64, compute_dtype=torch.float64)
    y1, S1 = chunk_scan(q[:, :, :128], k[:, :, :128], v[:, :, :128], g[:, :, :128], db, 64,
                        compute_dtype=torch.float64)
    y2, S2 = chunk_scan(q[:, :, 128:], k[:, :, 128:], v[:, :, 128:], g[:, :, 128:], db, 64,
                        initial_state=S1, compute_dtype=torch.float64)
    assert max_rel(torch.cat([y1, y2], 2), y) < 1e-12 and max_rel(S2, S) < 1e-12


def test_zero_decay_carries_only_previous_chunk():
    q, k, v, g = _small(T=192)
    y, S = chunk_scan(q, k, v, None, 0.0, 64, compute_dtype=torch.float64)
    Kc, Vc = k[:, :, 128:192], v[:, :, 128:192]
    assert max_rel(S, Kc.transpose(-1, -2) @ Vc) < 1e-12
    # chunk 2 sees exactly K_1^T V_1
    Q2 = q[:, :, 128:192]
    S1 = k[:, :, 64:128].transpose(-1, -2) @ v[:, :, 64:128]
    intra = (Q2 @ Kc.transpose(-1, -2)).tril() @ Vc
    assert max_rel(y[:, :, 128:192], intra + Q2 @ S1) < 1e-12


def test_corrected_equals_literal_on_first_chunk():
    q, k, v, g = _small(D=64, T=128)
    yl, _ = chunk_scan(q, k, v, g, 0.9, 64, mode="literal", compute_dtype=torch.float64)
    yc, _ = chunk_scan(q, k, v, g, 0.9, 64, mode="corrected", compute_dtype=torch.float64)
    assert max_rel(yc[:, :, :64], yl[:, :, :64]) < 1e-14
    assert max_rel(yc[:, :, 64:], yl[:, :, 64:]) > 1e-3


def test_gradcheck_corrected_float64():
    B, H, T, D = 1, 2, 20, 4
    g = torch.Generator().manual_seed(3)
    mk = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64, requires_grad=True)
    q, k, v, gt = mk(B, H, T, D), mk(B, H, T, D), mk(B, H, T, D), mk(B, H, T, D)
    dec = (torch.rand(H, D, generator=g, dtype=torch.float64) * 0.3 + 0.6).requires_grad_(True)
    s0 = mk(B, H, D, D)

    def f(q, k, v, gt, dec, s0):
        y, S = chunk_scan(q, k, v, gt, decay_bhd1(dec, B, H, D, torch.float64), 8,
                          initial_state=s0, compute_dtype=torch.float64)
        return y, S
    assert torch.autograd.gradcheck(f, (q, k, v, gt, dec, s0))


# --------------------------------------------------------------------------- #
# the kernels' backward algorithm (incl. forward-mode decay gradient) vs autograd
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("mode,D,T,gate,with_s0,with_dsT", [
    ("corrected", 16, 150, True, True, True),
    ("corrected", 16, 128, False, False, False),
    ("corrected", 32, 64, True, False, True),
    ("corrected", 8, 37, True, True, False),
    ("literal", 16, 64, True, True, True),
    ("literal", 16, 48, False, False, False),
])
def test_manual_backward_matches_autograd(mode, D, T, gate, with_s0, with_dsT):
    B, H = 2, 2
    C = 16
    g = torch.Generator().manual_seed(7)
    mk = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    q, k, v = mk(B, H, T, D), mk(B, H, T, D), mk(B, H, T, D)
    gt = torch.sigmoid(mk(B, H, T, D)) if gate else None
    dec = torch.rand(B, H, D, generator=g, dtype=torch.float64) * 0.4 + 0.55
    s0 = mk(B, H, D, D) * 0.1 if with_s0 else None
    dy = mk(B, H, T, D)
    dsT = mk(B, H, D, D) if with_dsT else None

    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    gl = gt.clone().requires_grad_(True) if gt is not None else None
    dl = dec.clone().requires_grad_(True)
    sl = s0.clone().requires_grad_(True) if s0 is not None else None
    y, S = chunk_scan(*leaves, gl, dl.unsqueeze(-1), C, initial_state=sl, mode=mode,
                      compute_dtype=torch.float64)
    loss = (y * dy).sum() + ((S * dsT).sum() if dsT is not None else 0.0)
    loss.backward()

    dq, dk, dv, dg, dd, ds0 = manual_backward(q, k, v, gt, dec, C, s0, dy, dsT, mode=mode)
    for name, got, ref in [("dq", dq, leaves[0].grad), ("dk", dk, leaves[1].grad),
                           ("dv", dv, leaves[2].grad), ("ddecay", dd, dl.grad)]:
        assert max_rel(got, ref) < 1e-10, (name, max_rel(got, ref))
    if gate:
        assert max_rel(dg, gl.grad) < 1e-10
    if with_s0:
        assert max_rel(ds0, sl.grad) < 1e-10


def test_seeded_workloads_shapes_and_layout():
    w = custom(2, 3, 130, 64)
    inp = make_inputs(w, seed=0)
    assert inp["q"].shape == (2, 3, 130, 64) and inp["q"].dtype == torch.bfloat16
    # [B, H, T, D] view over [B, T, H, D] memory, as the KDA layer produces
    assert inp["q"].stride() == (130 * 3 * 64, 64, 3 * 64, 1)
    assert inp["decay"].shape == (3, 64) and inp["s0"] is None
    w4 = WORKLOADS["10b-fwdbwd"]
    assert w4.s0_std == 0.02 and w4.decay_mean == 4.0


# --------------------------------------------------------------------------- #
# per-step (docstring) semantics: the chunked restatement the kernels run
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("B,H,T,D,decay,gate,with_s0", [
    (1, 2, 150, 8, 0.9, True, True),       # ragged last chunk
    (2, 1, 64, 16, 0.5, False, False),
    (1, 2, 200, 8, 0.125, True, True),     # smallest supported decay
    (1, 1, 129, 8, 1.0, True, False),
    (1, 3, 70, 4, "head", True, True),     # one decay per head
])
def test_per_step_chunked_form_and_backward_match_the_recurrence(B, H, T, D, decay, gate, with_s0):
    from oracle.kda_oracle import per_step_chunk_scan, per_step_manual_backward, per_step_recurrence
    g = torch.Generator().manual_seed(21)
    q, k, v, gt = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64) for _ in range(4))
    gt = gt if gate else None
    dec = torch.tensor([0.9, 0.5, 0.99], dtype=torch.float64) if decay == "head" else decay
    s0 = torch.randn(B, H, D, D, generator=g, dtype=torch.float64) if with_s0 else None
    y1, s1 = per_step_recurrence(q, k, v, gt, dec, s0)
    y2, s2 = per_step_chunk_scan(q, k, v, gt, dec, 64, s0)
    assert max_rel(y2, y1) < 1e-12 and max_rel(s2, s1) < 1e-12
    leaves = [t.clone().requires_grad_() for t in (q, k, v)]
    gl = gt.clone().requires_grad_() if gt is not None else None
    sl = s0.clone().requires_grad_() if s0 is not None else None
    y, s = per_step_recurrence(*leaves, gl, dec, sl)
    dy, dsT = torch.randn_like(y), torch.randn_like(s)
    ((y * dy).sum() + (s * dsT).sum()).backward()
    dq, dk, dv, dg, ds0 = per_step_manual_backward(q, k, v, gt, dec, 64, s0, dy, dsT)
    pairs = [(dq, leaves[0].grad), (dk, leaves[1].grad), (dv, leaves[2].grad)]
    if gl is not None:
        pairs.append((dg, gl.grad))
    if sl is not None:
        pairs.append((ds0, sl.grad))
    for got, ref in pairs:
        assert max_rel(got, ref) < 1e-12


def test_per_step_recurrence_is_the_docstring_loop():
    """s_t = a s_{t-1} + k_t^T v_t, o_t = q_t s_t, y_t = g_t o_t (kernels/kda_kernel.py:8-11), by hand."""
    from oracle.kda_oracle import per_step_recurrence
    q = torch.tensor([[[[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]]]])
    k = torch.tensor([[[[1.0, 0.0], [0.0, 1.0], [1.0, 0.0]]]])
    v = torch.tensor([[[[2.0, 0.0], [0.0, 3.0], [1.0, 1.0]]]])
    y, s = per_step_recurrence(q, k, v, None, 0.5, None)
    # s_0 = [[2,0],[0,0]]; s_1 = [[1,0],[0,3]]; s_2 = [[1.5,1],[0,1.5]]
    assert torch.allclose(s[0, 0], torch.tensor([[1.5, 1.0], [0.0, 1.5]], dtype=torch.float64))
    assert torch.allclose(y[0, 0], torch.tensor([[2.0, 0.0], [0.0, 3.0], [1.5, 2.5]], dtype=torch.float64))
