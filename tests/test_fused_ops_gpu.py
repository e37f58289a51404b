"""sm_100a fused ops (include/st_fused_ops.h) against plain PyTorch fp32.

The references restate kernels/fused_ops.py's torch paths
(silu_mul_torch :96-97, rmsnorm_residual_torch :160-167,
cross_entropy_torch :289-294) in fp32; gradients come from autograd through
them.  Tolerance: normwise max|x - ref| / max|ref| <= 2e-2 for 16-bit
results, 1e-3 for the fp32 loss.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle.kda_oracle import max_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL_LOWP = 2e-2
TOL_F32 = 1e-3


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _leaf(t):
    return t.detach().clone().requires_grad_(True)


@pytest.mark.parametrize("shape,dtype", [((2, 5, 101), torch.bfloat16), ((64, 1024), torch.bfloat16),
                                         ((3, 7, 256), torch.float16), ((1, 13), torch.bfloat16)])
def test_silu_mul_forward_backward(shape, dtype):
    from simpletrain_b200.fused_ops import fused_silu_mul
    g = torch.Generator().manual_seed(0)
    a = torch.randn(shape, generator=g).to(dtype).to(DEV)
    b = torch.randn(shape, generator=g).to(dtype).to(DEV)
    dout = torch.randn(shape, generator=g).to(dtype).to(DEV)
    a1, b1 = _leaf(a), _leaf(b)
    out = fused_silu_mul(a1, b1)
    assert out.dtype == dtype and out.shape == a.shape
    out.backward(dout)
    a2, b2 = _leaf(a.float()), _leaf(b.float())
    ref = F.silu(a2) * b2
    ref.backward(dout.float())
    assert max_rel(out.float().cpu(), ref.detach().cpu()) <= TOL_LOWP
    assert max_rel(a1.grad.float().cpu(), a2.grad.cpu()) <= TOL_LOWP
    assert max_rel(b1.grad.float().cpu(), b2.grad.cpu()) <= TOL_LOWP


@pytest.mark.parametrize("N,D,dtype", [(333, 1024, torch.bfloat16), (17, 100, torch.bfloat16),
                                       (64, 2048, torch.float16), (45, 2560, torch.bfloat16),
                                       (9, 8208, torch.bfloat16)])
def test_rmsnorm_residual_forward_backward(N, D, dtype):
    from simpletrain_b200.fused_ops import fused_rmsnorm_residual
    g = torch.Generator().manual_seed(1)
    x = torch.randn(N, D, generator=g).to(dtype).to(DEV)
    r = torch.randn(N, D, generator=g).to(dtype).to(DEV)
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype).to(DEV)
    dy = torch.randn(N, D, generator=g).to(dtype).to(DEV)
    x1, r1, w1 = _leaf(x), _leaf(r), _leaf(w)
    out = fused_rmsnorm_residual(x1, r1, w1, 1e-6)
    out.backward(dy)
    x2, r2, w2 = _leaf(x.float()), _leaf(r.float()), _leaf(w.float())
    ref = x2 * torch.rsqrt(x2.pow(2).mean(-1, keepdim=True) + 1e-6) * w2 + r2
    ref.backward(dy.float())
    assert max_rel(out.float().cpu(), ref.detach().cpu()) <= TOL_LOWP
    for got, exp in ((x1.grad, x2.grad), (r1.grad, r2.grad), (w1.grad, w2.grad)):
        assert max_rel(got.float().cpu(), exp.cpu()) <= TOL_LOWP


@pytest.mark.parametrize("N,V,dtype", [(64, 32000, torch.bfloat16), (37, 1001, torch.bfloat16),
                                       (8, 50304, torch.float16)])
def test_cross_entropy_forward_backward(N, V, dtype):
    from simpletrain_b200.fused_ops import cross_entropy_loss, fused_cross_entropy
    g = torch.Generator().manual_seed(2)
    logits = (3 * torch.randn(N, V, generator=g)).to(dtype).to(DEV)
    labels = torch.randint(0, V, (N,), generator=g).to(DEV)
    l1 = _leaf(logits)
    loss, probs = fused_cross_entropy(l1, labels)
    loss.backward()
    l2 = _leaf(logits.float())
    ref = F.cross_entropy(l2, labels)
    ref.backward()
    assert abs(loss.item() - ref.item()) <= TOL_F32 * max(1.0, abs(ref.item()))
    assert probs.dtype == dtype and probs.shape == logits.shape
    assert max_rel(probs.float().cpu(), torch.softmax(logits.float(), -1).cpu()) <= TOL_LOWP
    assert max_rel(l1.grad.float().cpu(), l2.grad.cpu()) <= TOL_LOWP
    assert abs(cross_entropy_loss(logits, labels).item() - ref.item()) <= TOL_F32 * max(1.0, abs(ref.item()))


def test_install_routes_fused_ops_imports():
    import sys
    import simpletrain_b200
    simpletrain_b200.install()
    from kernels.fused_ops import fused_cross_entropy, fused_rmsnorm_residual, fused_silu_mul  # noqa: F401
    assert sys.modules["kernels.fused_ops"].__name__ == "simpletrain_b200.fused_ops"
