"""Opt-in fused forward for SimpleTrain's KDA layer.

``KimiDeltaAttention.forward`` (``models/kimi_k3.py:94-125``) runs four
projection GEMMs, reads the mean decay back to the host with ``.item()``
(``:109``, one device-to-host sync per layer per step) and then calls the scan.
``fused_forward`` computes the same function of the same parameters with

* one projection GEMM, ``x @ cat(W_q, W_k, W_v, W_g)^T``: x is read once instead
  of four times, and q, k, v, g are ``[B, H, T, Dh]`` views of its output that
  the scan's TMA loads read in place (token stride ``4 H Dh``);
* the per-head decay's mean handed to the scan as a device tensor, so nothing
  waits for the GPU;
* the scan's y in ``[B, T, H, Dh]`` memory order, so the head scale keeps that
  order and the final ``transpose(1, 2).contiguous()`` copies nothing.

Gradients reach the four projection weights through the concatenation, and the
head scale's gradient reaches ``log_decay`` exactly as in the layer (the decay
passed to the scan is detached there too, ``:105``).  The scan's state-update
semantics are those of the drop-in ``kernels.kda_kernel``
(``simpletrain_b200.kda_kernel.SEMANTICS``).

``install_fused_layer()`` replaces ``KimiDeltaAttention.forward`` with it; the
module, its parameters and its call signature stay as they are.
"""
from __future__ import annotations

import math
import sys

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import kda_kernel


def _use_triton(layer) -> bool:
    """The layer's ``use_triton`` setting: ``cfg.use_triton`` on SimpleTrain's
    module (``models/kimi_k3.py:117``), the attribute on ``KDALayer``."""
    cfg = getattr(layer, "cfg", None)
    if cfg is not None and hasattr(cfg, "use_triton"):
        return bool(cfg.use_triton)
    return bool(getattr(layer, "use_triton", True))


def fused_forward(self, x: torch.Tensor) -> torch.Tensor:
    """``KimiDeltaAttention.forward`` with one projection GEMM and no host sync: [B, T, D] -> [B, T, D]."""
    B, T, _ = x.shape
    H, Dh = self.n_heads, self.d_head
    w = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.g_proj.weight], 0)
    # unbind: its backward is one stack of the four gradients (indexing would
    # zero-fill and sum four full-size buffers)
    qkvg = F.linear(x, w).view(B, T, 4, H, Dh).unbind(2)
    dt = self._dtype()
    q, k, v, g = (t.transpose(1, 2).to(dt) for t in qkvg)   # [B, H, T, Dh] views
    decay = torch.exp(self.log_decay).clamp(min=1e-3, max=0.999).detach().mean()   # stays on the device
    o = kda_kernel.kda_chunked_scan(q, k, v, gate=g, decay=decay, chunk_size=self.chunk,
                                    use_triton=_use_triton(self))   # [B, H, T, Dh]
    head_scale = torch.exp(self.log_decay).clamp(min=1e-3, max=0.999)
    o = o * head_scale.view(1, H, 1, 1).to(o.dtype)
    return self.o_proj(o.transpose(1, 2).contiguous().view(B, T, H * Dh))


def install_fused_layer() -> bool:
    """Replace ``models.kimi_k3.KimiDeltaAttention.forward`` with ``fused_forward``.

    Returns False (and changes nothing) when ``models.kimi_k3`` cannot be imported.
    """
    try:
        import importlib
        model = sys.modules.get("models.kimi_k3") or importlib.import_module("models.kimi_k3")
    except ImportError:
        return False
    model.KimiDeltaAttention.forward = fused_forward
    return True


def unfused_forward(self, x: torch.Tensor) -> torch.Tensor:
    """The layer's forward as SimpleTrain structures it (``models/kimi_k3.py:94-125``):
    four projection GEMMs, the mean decay read back with ``.item()``, then the same
    scan.  For comparisons with ``fused_forward`` on the same module."""
    B, T, _ = x.shape
    H, Dh = self.n_heads, self.d_head
    dt = self._dtype()
    q, k, v, g = (p(x).view(B, T, H, Dh).transpose(1, 2).to(dt)
                  for p in (self.q_proj, self.k_proj, self.v_proj, self.g_proj))
    decay = float(torch.exp(self.log_decay).clamp(min=1e-3, max=0.999).detach().mean().item())
    o = kda_kernel.kda_chunked_scan(q, k, v, gate=g, decay=decay, chunk_size=self.chunk,
                                    use_triton=_use_triton(self))
    head_scale = torch.exp(self.log_decay).clamp(min=1e-3, max=0.999)
    o = o * head_scale.view(1, H, 1, 1).to(o.dtype)
    return self.o_proj(o.transpose(1, 2).contiguous().view(B, T, H * Dh))


class KDALayer(nn.Module):
    """A KDA layer with the parameters of SimpleTrain's ``KimiDeltaAttention``
    (``models/kimi_k3.py:72-92``: ``q_proj``, ``k_proj``, ``v_proj``, ``g_proj``,
    ``o_proj`` without bias, per-head ``log_decay``), so state dicts load either
    way, running ``fused_forward``."""

    def __init__(self, d_model: int, n_heads: int, d_head: int, chunk_size: int = 64,
                 decay_base: float = 0.99, dtype: torch.dtype = torch.bfloat16,
                 use_triton: bool = True):
        super().__init__()
        self.n_heads, self.d_head, self.chunk = n_heads, d_head, chunk_size
        self.use_triton = use_triton
        self.inner = n_heads * d_head
        self._dt = dtype
        self.q_proj = nn.Linear(d_model, self.inner, bias=False)
        self.k_proj = nn.Linear(d_model, self.inner, bias=False)
        self.v_proj = nn.Linear(d_model, self.inner, bias=False)
        self.g_proj = nn.Linear(d_model, self.inner, bias=False)
        self.o_proj = nn.Linear(self.inner, d_model, bias=False)
        self.log_decay = nn.Parameter(torch.full((n_heads,), math.log(decay_base)))
        nn.init.zeros_(self.g_proj.weight)

    def _dtype(self) -> torch.dtype:
        return self._dt

    forward = fused_forward
