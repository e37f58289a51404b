"""The opt-in fused KDA layer forward against the layer's own structure.

``fused_forward`` (one projection GEMM, decay kept on the device, y in
[B, T, H, Dh] order) must compute the same outputs and parameter gradients as
``unfused_forward`` (four GEMMs and the ``.item()`` of models/kimi_k3.py:94-125)
on the same module, and must not synchronise with the host.  Tolerance:
normwise max-rel 2e-2 (bf16).
"""
import pytest
import torch

from oracle.kda_oracle import max_rel
from simpletrain_b200 import device_status
from simpletrain_b200.kda_layer import KDALayer, fused_forward, unfused_forward

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert device_status() == 0


def _layer(d_model, H, Dh, seed):
    torch.manual_seed(seed)
    layer = KDALayer(d_model, H, Dh).to(DEV).to(torch.bfloat16)
    with torch.no_grad():   # a live gate and per-head decays, so every gradient is non-trivial
        layer.g_proj.weight.normal_(0.0, d_model ** -0.5)
        layer.log_decay.copy_(torch.log(torch.linspace(0.9, 0.99, H)))
    layer.log_decay.data = layer.log_decay.data.float()
    return layer


@pytest.mark.parametrize("d_model,H,Dh,T", [(256, 4, 64, 256), (256, 2, 128, 200)])
def test_fused_layer_matches_the_layer_structure(d_model, H, Dh, T):
    layer = _layer(d_model, H, Dh, seed=3)
    x = torch.randn(2, T, d_model, device=DEV, dtype=torch.bfloat16)
    dy = torch.randn(2, T, d_model, device=DEV, dtype=torch.bfloat16)
    results = []
    for fwd in (unfused_forward, fused_forward):
        layer.zero_grad()
        xl = x.clone().requires_grad_(True)
        y = fwd(layer, xl)
        (y.float() * dy.float()).sum().backward()
        grads = {n: p.grad.clone() for n, p in layer.named_parameters()}
        results.append((y.detach(), xl.grad.clone(), grads))
    (y0, dx0, g0), (y1, dx1, g1) = results
    assert max_rel(y1.float(), y0.float()) <= TOL
    assert max_rel(dx1.float(), dx0.float()) <= TOL
    for n in g0:
        assert max_rel(g1[n].float(), g0[n].float()) <= TOL, n


def test_fused_layer_does_not_sync_with_the_host():
    layer = _layer(256, 2, 128, seed=4)
    x = torch.randn(2, 128, 256, device=DEV, dtype=torch.bfloat16)
    fused_forward(layer, x)      # warm up (library loads, workspace queries)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        y = fused_forward(layer, x)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.set_sync_debug_mode("error")
    try:
        with pytest.raises(RuntimeError):
            unfused_forward(layer, x)   # the .item() of the layer's own structure
    finally:
        torch.cuda.set_sync_debug_mode("default")
    assert y.shape == x.shape


def test_scan_output_keeps_the_fused_projection_order():
    """q, k, v, g as views of one [B, T, 4, H, Dh] projection: y comes back in
    [B, T, H, Dh] memory, so the layer's transpose + contiguous() is free."""
    from simpletrain_b200 import kda_chunked_scan
    B, T, H, Dh = 2, 128, 4, 64
    qkvg = torch.randn(B, T, 4, H, Dh, device=DEV, dtype=torch.bfloat16)
    q, k, v, g = (qkvg[:, :, i].transpose(1, 2) for i in range(4))
    y = kda_chunked_scan(q, k, v, gate=g, decay=torch.tensor(0.95, device=DEV))
    assert y.transpose(1, 2).is_contiguous()
