"""Drop-in for SimpleTrain's ``kernels/kda_kernel.py``.

Same public names and argument meaning as the reference module:

* ``kda_chunked_scan(q, k, v, gate=None, decay=0.99, chunk_size=64,
  use_triton=True) -> y``                      (``kernels/kda_kernel.py:303-328``)
* ``kda_chunked_scan_triton(q, k, v, gate=None, decay=0.99, chunk_size=64)``
                                               (``kernels/kda_kernel.py:195-238``)
* ``_supported_arch()``                        (``kernels/kda_kernel.py:58-67``)

Both scan functions run the sm_100a kernels through the ``kda_b200`` custom
op (there is one implementation and no CPU path).  The result keeps the
reference's conventions: y has q's dtype, shape and memory order (``:263``),
the state is not returned (``:297``), and ``decay`` is a float or a tensor
broadcasting as ``[B, H, D, 1]`` against the state (``:295``).

Input dtypes follow the reference's dispatch on an sm_100 GPU (``:303-328``):
with ``use_triton=True`` (the model's default, ``config.py:64``) fp16/bf16
inputs run and fp32 inputs raise ``AssertionError``, because the reference's
Triton wrapper asserts before its fallback (``:204``); with
``use_triton=False`` the reference runs its fp32 torch loop, which takes any
floating dtype, and so does this module: fp32 inputs are rounded to bf16 for
the tensor-core scan (fp32 products, sums and state, as for bf16 inputs) and y
comes back in fp32, within the bf16 tolerance (normwise 2e-2) of the
reference's fp32 result.  Gradients flow through the roundings.

State-update semantics (module attribute ``SEMANTICS``, or the environment
variable ``KDA_B200_SEMANTICS`` read at import):

* ``"auto"`` (default) -- the reference's literal ``K V^T`` update
  (``:294``) wherever the reference itself runs (D == chunk_size, and every
  chunk but the last full or the last of length 1), so results match the
  reference on those shapes; the ``K^T V`` update everywhere else (D=128,
  where the reference raises).
* ``"literal"`` -- always the reference's update; raises like the reference
  (``RuntimeError``, same message) when D != chunk_size.
* ``"corrected"`` -- always ``K^T V``.
* ``"per_step"`` -- the per-token recurrence of the reference's docstring
  (``:8-11``) and Triton kernel (``:134-180``), ``s_t = decay s_{t-1} +
  k_t^T v_t``, with one decay per (batch, head) in [0.125, 1].

Errors: fp32 inputs with ``use_triton=True`` (or through
``kda_chunked_scan_triton``) raise ``AssertionError`` like the reference
(``:204``); other dtypes raise ``TypeError``; CPU tensors raise
``RuntimeError`` (there is no CPU path: the reference would run its torch
loop on the CPU, this module serves only the B200 kernels).

``install()`` makes ``import kernels.kda_kernel`` (and an already imported
``models.kimi_k3``) resolve to this module, so ``models/kimi_k3.py`` and
``train.py`` run unchanged.
"""
from __future__ import annotations

import os
import sys
from typing import Optional, Union

import torch

from .ops import _validate, kda_chunk

SEMANTICS = os.environ.get("KDA_B200_SEMANTICS", "auto")


def _supported_arch() -> bool:
    """True iff the current CUDA device is a B200-class sm_100 part."""
    if not torch.cuda.is_available():
        return False
    try:
        return torch.cuda.get_device_capability() == (10, 0)
    except Exception:
        return False


def _use_literal(D: int, T: int, chunk_size: int) -> bool:
    mode = SEMANTICS
    if mode == "literal":
        return True
    if mode in ("corrected", "per_step"):
        return False
    if mode != "auto":
        raise ValueError(f"SEMANTICS must be 'auto', 'literal', 'corrected' or 'per_step', got {mode!r}")
    return D == chunk_size and (T % chunk_size) in (0, 1)


def _per_step_decay_arg(decay: Union[float, torch.Tensor], B: int, H: int):
    """A float, or a tensor broadcasting as [B, H, 1, 1] (one decay per head), as [B, H, 1]."""
    if not torch.is_tensor(decay):
        return float(decay)
    return torch.broadcast_to(decay.float(), (B, H, 1, 1)).reshape(B, H, 1)


def _decay_arg(decay: Union[float, torch.Tensor], B: int, H: int, D: int):
    """The reference's decay broadcast ([B, H, D, 1] against the state) as [B, H, D]."""
    if not torch.is_tensor(decay):
        return float(decay)
    d = decay.float()
    if d.dim() == 0:
        return d.reshape(1, 1, 1).expand(B, H, D)
    if d.shape[-1] != 1 and D != 1:
        raise NotImplementedError(
            "decay tensors must broadcast as [B, H, D, 1] (one factor per key-channel row)")
    return torch.broadcast_to(d, (B, H, D, 1)).squeeze(-1)


def _scan16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gate: Optional[torch.Tensor],
            decay: Union[float, torch.Tensor], chunk_size: int) -> torch.Tensor:
    """The sm_100a scan on fp16/bf16 inputs, in the semantics ``SEMANTICS`` picks."""
    _validate(q, k, v, gate, chunk_size)
    B, H, T, D = q.shape
    if SEMANTICS == "per_step":
        y, _ = kda_chunk(q, k, v, gate, _per_step_decay_arg(decay, B, H), None, chunk_size,
                         output_final_state=False, per_step=True)
        return y
    literal = _use_literal(D, T, chunk_size)
    y, _ = kda_chunk(q, k, v, gate, _decay_arg(decay, B, H, D), None, chunk_size,
                     reference_exact=literal, output_final_state=False)
    return y


def kda_chunked_scan_triton(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            gate: Optional[torch.Tensor] = None, decay: float = 0.99,
                            chunk_size: int = 64) -> torch.Tensor:
    """Run the scan on the sm_100a kernels; returns y of shape ``[B, H, T, D]``.

    Takes fp16/bf16 inputs only, as the reference's wrapper asserts (``:204``)."""
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise AssertionError("KDA sm_100a kernel requires fp16/bf16")
    return _scan16(q, k, v, gate, decay, chunk_size)


def kda_chunked_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     gate: Optional[torch.Tensor] = None, decay: float = 0.99,
                     chunk_size: int = 64, use_triton: bool = True) -> torch.Tensor:
    """SimpleTrain's KDA dispatch, served by the sm_100a kernels.

    ``use_triton=True``: fp16/bf16 only (fp32 raises ``AssertionError``, as the
    reference's wrapper does on an sm_100 GPU).  ``use_triton=False``: the
    reference's torch loop takes fp32 too; fp32 inputs run here on bf16-rounded
    copies and y is returned in fp32."""
    if use_triton or q.dtype in (torch.float16, torch.bfloat16):
        return kda_chunked_scan_triton(q, k, v, gate, decay, chunk_size)
    if q.dtype != torch.float32:
        raise TypeError(f"KDA scan takes fp32, fp16 or bf16 inputs, got {q.dtype}")
    if q.device.type != "cuda":
        raise RuntimeError("the KDA sm_100a kernels need CUDA tensors (there is no CPU path)")
    lo = torch.bfloat16
    y = _scan16(q.to(lo), k.to(lo), v.to(lo), gate.to(lo) if gate is not None else None,
                decay, chunk_size)
    return y.to(q.dtype)


def install() -> None:
    """Route SimpleTrain's ``kernels.kda_kernel`` imports to this module and
    ``kernels.fused_ops`` imports to ``simpletrain_b200.fused_ops``.

    Call before importing ``models.kimi_k3``; an already imported
    ``models.kimi_k3`` has its ``kda_chunked_scan`` and fused-op names rebound too.
    """
    import importlib
    import types

    me = sys.modules[__name__]
    from . import fused_ops as fo
    try:
        pkg = importlib.import_module("kernels")
    except ModuleNotFoundError:  # SimpleTrain not on sys.path: a bare package to hang the modules on
        pkg = types.ModuleType("kernels")
        pkg.__path__ = []
        sys.modules["kernels"] = pkg
    sys.modules["kernels.kda_kernel"] = me
    sys.modules["kernels.fused_ops"] = fo
    setattr(pkg, "kda_kernel", me)
    setattr(pkg, "fused_ops", fo)
    model = sys.modules.get("models.kimi_k3")
    if model is not None:
        setattr(model, "kda_chunked_scan", kda_chunked_scan)
        for name in ("fused_silu_mul", "fused_rmsnorm_residual", "fused_cross_entropy"):
            setattr(model, name, getattr(fo, name))
