"""sm_100a replacements for SimpleTrain's ``kernels/fused_ops.py``, with autograd.

Same names, arguments and results as the reference module, so
``install()`` can map ``kernels.fused_ops`` here; the difference is that
every op runs the library's CUDA kernels (``include/st_fused_ops.h``) and is
differentiable, where the reference's Triton outputs carry no autograd graph
(``kernels/fused_ops.py:83-93, 148-157, 272-286``) and its torch fallbacks
run plain PyTorch.  ``use_triton`` is accepted and ignored; CPU tensors are
rejected (there is no CPU path).

* ``fused_silu_mul(a, b)`` -> ``silu(a) * b`` in a's dtype (any shape).
* ``fused_rmsnorm_residual(x, residual, weight, eps)`` ->
  ``x * rsqrt(mean(x^2) + eps) * weight + residual`` over the last dimension.
* ``fused_cross_entropy(logits[N, V], labels[N])`` -> ``(mean NLL, softmax)``;
  gradients flow through the loss (the softmax output is a plain tensor, as
  in the reference, which returns it for inspection / distillation).
"""
from __future__ import annotations

import torch

from . import ops as _ops  # noqa: F401  (loads the library that defines the st_b200 ops)

Tensor = torch.Tensor


def _need_cuda(*ts: Tensor):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("the sm_100a fused ops need CUDA tensors (there is no CPU path)")


# --------------------------------------------------------------------- silu*mul
@torch.library.register_fake("st_b200::silu_mul")
def _(a, b):
    return torch.empty_like(a)


@torch.library.register_fake("st_b200::silu_mul_bwd")
def _(a, b, dout):
    return torch.empty_like(a), torch.empty_like(b)


def _silu_setup(ctx, inputs, output):
    a, b = inputs
    ctx.save_for_backward(a, b)


def _silu_backward(ctx, dout):
    a, b = ctx.saved_tensors
    da, db = torch.ops.st_b200.silu_mul_bwd(a, b, dout)
    return da.view_as(a), db.view_as(b)


torch.library.register_autograd("st_b200::silu_mul", _silu_backward, setup_context=_silu_setup)


def silu_mul_triton(a: Tensor, b: Tensor) -> Tensor:
    """silu(a) * b on sm_100a (the reference's Triton entry point name)."""
    _need_cuda(a, b)
    if a.shape != b.shape:
        raise AssertionError("silu_mul: a and b must have the same shape")
    return torch.ops.st_b200.silu_mul(a, b).view(a.shape)


def fused_silu_mul(a: Tensor, b: Tensor, *, use_triton: bool = True) -> Tensor:
    """kernels/fused_ops.py:100-109, differentiable."""
    return silu_mul_triton(a, b)


# ------------------------------------------------------------- RMSNorm + residual
@torch.library.register_fake("st_b200::rmsnorm_residual")
def _(x, residual, weight, eps):
    return torch.empty_like(x), x.new_empty(x.shape[:-1], dtype=torch.float32)


@torch.library.register_fake("st_b200::rmsnorm_residual_bwd")
def _(x, weight, rstd, dy):
    return torch.empty_like(x), x.new_empty((x.shape[-1],), dtype=torch.float32)


def _rms_setup(ctx, inputs, output):
    x, residual, weight, eps = inputs
    _, rstd = output
    ctx.save_for_backward(x, weight, rstd)
    ctx.res_dtype = residual.dtype
    ctx.w_dtype = weight.dtype


def _rms_backward(ctx, dy, _drstd):
    x, weight, rstd = ctx.saved_tensors
    dx, dw = torch.ops.st_b200.rmsnorm_residual_bwd(x, weight, rstd, dy)
    return dx.view_as(x), dy.to(ctx.res_dtype), dw.to(ctx.w_dtype), None


torch.library.register_autograd("st_b200::rmsnorm_residual", _rms_backward, setup_context=_rms_setup)


def rmsnorm_residual_triton(x: Tensor, residual: Tensor, weight: Tensor, eps: float) -> Tensor:
    """RMSNorm + residual on sm_100a (the reference's Triton entry point name)."""
    _need_cuda(x, residual, weight)
    out, _ = torch.ops.st_b200.rmsnorm_residual(x, residual, weight, float(eps))
    return out.view(x.shape)


def fused_rmsnorm_residual(x: Tensor, residual: Tensor, weight: Tensor, eps: float, *,
                           use_triton: bool = True) -> Tensor:
    """kernels/fused_ops.py:170-181, differentiable in x, residual and weight."""
    return rmsnorm_residual_triton(x, residual, weight, eps)


# ------------------------------------------------------------------ cross-entropy
@torch.library.register_fake("st_b200::cross_entropy")
def _(logits, labels, want_probs):
    N = logits.shape[0]
    f32 = torch.float32
    probs = torch.empty_like(logits) if want_probs else logits.new_empty((0,))
    return logits.new_empty((N,), dtype=f32), logits.new_empty((N,), dtype=f32), probs


@torch.library.register_fake("st_b200::cross_entropy_bwd")
def _(logits, labels, lse, dloss):
    return torch.empty_like(logits)


def _ce_setup(ctx, inputs, output):
    logits, labels, _ = inputs
    _, lse, _ = output
    ctx.save_for_backward(logits, labels, lse)


def _ce_backward(ctx, dloss, _dlse, dprobs):
    if dprobs is not None and dprobs.numel() and bool(dprobs.abs().sum() > 0):
        raise NotImplementedError("gradients through the softmax output are not supported")
    logits, labels, lse = ctx.saved_tensors
    return torch.ops.st_b200.cross_entropy_bwd(logits, labels, lse, dloss), None, None


torch.library.register_autograd("st_b200::cross_entropy", _ce_backward, setup_context=_ce_setup)


def cross_entropy_triton(logits: Tensor, labels: Tensor) -> tuple[Tensor, Tensor]:
    """Returns (mean_loss, softmax_probs[N, V]) like kernels/fused_ops.py:266-286."""
    _need_cuda(logits, labels)
    loss_rows, _, probs = torch.ops.st_b200.cross_entropy(logits, labels, True)
    return loss_rows.mean(), probs


def cross_entropy_loss(logits: Tensor, labels: Tensor) -> Tensor:
    """Mean NLL only: skips writing the [N, V] softmax the reference API returns."""
    _need_cuda(logits, labels)
    loss_rows, _, _ = torch.ops.st_b200.cross_entropy(logits, labels, False)
    return loss_rows.mean()


def fused_cross_entropy(logits: Tensor, labels: Tensor, *, use_triton: bool = True) -> tuple[Tensor, Tensor]:
    """kernels/fused_ops.py:297-307, differentiable through the loss."""
    return cross_entropy_triton(logits, labels)


def _supported_arch() -> bool:
    """True on sm_100 devices (the only ones these kernels are built for)."""
    return torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
