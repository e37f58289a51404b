"""Seeded synthetic KDA workloads.

SimpleTrain's KDA layer (``models/kimi_k3.py:94-125``) feeds the scan with
``[B, H, T, D]`` views of the q/k/v/g projections.  There is no public dataset
on this path, so every workload here is synthetic with fixed distributions:

* q, k ~ N(0, 1), then L2-normalised over the head dimension D
* v ~ N(0, 1)
* g = sigmoid(N(0, 1))                       (output gate)
* decay = sigmoid(N(3, 1)) per key channel, shape [H, D]
  (sigmoid(N(4, 1)) for the long-context shape)
* initial state zero, except the long-context shape: N(0, 0.02) fp32 [B, H, D, D]
* upstream gradient dy ~ N(0, 1)

All tensors are drawn on the CPU from one ``torch.Generator`` seeded with
``seed`` in the fixed order q, k, v, g, decay, s0, dy, so the same seed gives
the same bytes on every machine running the same torch build.

Shapes follow SimpleTrain's model variants (``config.py:107-173``): the 100m
variant has 8 heads of 64, 1b has 10 heads of 128, 7b 24 heads of 128 and 10b
28 heads of 128; chunk length is ``kda_chunk_size = 64`` (``config.py:37``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    T: int
    D: int
    dtype: torch.dtype
    backward: bool
    decay_mean: float = 3.0
    s0_std: float = 0.0
    chunk: int = 64

    @property
    def tokens(self) -> int:
        return self.B * self.T

    def describe(self) -> Dict[str, object]:
        return {
            "workload": self.name,
            "B": self.B,
            "H": self.H,
            "T": self.T,
            "D_head": self.D,
            "chunk": self.chunk,
            "pass": "fwd+bwd" if self.backward else "fwd",
            "dtype": {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[self.dtype],
        }


WORKLOADS: Dict[str, Workload] = {
    # CPU-sized forward, fp32: the reference torch path's own runnable case.
    "cpu-fwd-f32": Workload("cpu-fwd-f32", 2, 8, 512, 64, torch.float32, False),
    # 100m-variant shape, forward only.
    "100m-fwd": Workload("100m-fwd", 16, 8, 2048, 64, torch.bfloat16, False),
    # 1b-variant shape, forward + backward (the headline workload).
    "1b-fwdbwd": Workload("1b-fwdbwd", 16, 10, 2048, 128, torch.bfloat16, True),
    # 7b-variant shape, forward + backward.
    "7b-fwdbwd": Workload("7b-fwdbwd", 8, 24, 4096, 128, torch.bfloat16, True),
    # 10b-variant long context, non-zero initial state, slower decay.
    "10b-fwdbwd": Workload("10b-fwdbwd", 1, 28, 32768, 128, torch.bfloat16, True,
                           decay_mean=4.0, s0_std=0.02),
}


def custom(B: int, H: int, T: int, D: int, dtype=torch.bfloat16, backward=True,
           decay_mean: float = 3.0, s0_std: float = 0.0, chunk: int = 64) -> Workload:
    return Workload(f"custom-B{B}H{H}T{T}D{D}", B, H, T, D, dtype, backward,
                    decay_mean, s0_std, chunk)


def make_inputs(w: Workload, seed: int = 0, device: Optional[str] = None) -> Dict[str, torch.Tensor]:
    """Draw the seeded inputs of workload ``w``.

    Returns a dict with q, k, v, g (``[B, H, T, D]`` in ``w.dtype``), decay
    (``[H, D]`` fp32), s0 (``[B, H, D, D]`` fp32 or None) and dy
    (``[B, H, T, D]`` in ``w.dtype``).  q/k/v/g/dy are ``[B, H, T, D]`` views
    over ``[B, T, H, D]`` memory, which is how the KDA layer hands them over
    (``models/kimi_k3.py:99-102``).
    """
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    B, H, T, D = w.B, w.H, w.T, w.D

    def bthd(x: torch.Tensor) -> torch.Tensor:
        # drawn as [B, T, H, D] (the projection's memory order), viewed [B, H, T, D]
        return x.to(w.dtype).transpose(1, 2)

    def normal(*shape, mean=0.0, std=1.0):
        return torch.randn(*shape, generator=gen, dtype=torch.float32) * std + mean

    q = normal(B, T, H, D)
    q = q / q.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    k = normal(B, T, H, D)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    v = normal(B, T, H, D)
    g = torch.sigmoid(normal(B, T, H, D))
    decay = torch.sigmoid(normal(H, D, mean=w.decay_mean))
    s0 = normal(B, H, D, D, std=w.s0_std) if w.s0_std > 0 else None
    dy = normal(B, T, H, D) if w.backward else None

    out = {
        "q": bthd(q), "k": bthd(k), "v": bthd(v), "g": bthd(g),
        "decay": decay, "s0": s0, "dy": bthd(dy) if dy is not None else None,
    }
    if device is not None:
        out = {n: (t.to(device) if t is not None else None) for n, t in out.items()}
        # .to() on a strided view keeps the [B, T, H, D] memory order
    return out


def layer_params(d_model: int, n_heads: int, d_head: int, seed: int = 0) -> Dict[str, torch.Tensor]:
    """Seeded fp32 parameters of one KDA layer, keyed by SimpleTrain's names.

    ``KimiDeltaAttention`` (``models/kimi_k3.py:81-89``) holds ``q_proj``,
    ``k_proj``, ``v_proj``, ``g_proj`` and ``o_proj`` (bias-free Linear) and a
    per-head ``log_decay``.  Weights are N(0, 1/fan_in); the gate projection is
    drawn too (the layer zero-initialises it, ``:92``, which would make every
    output zero); ``log_decay = log(U(0.9, 0.99))`` per head, so the scan's mean
    decay and the per-head scale (``:105-122``) both vary.  Drawn in the fixed
    order q, k, v, g, o, log_decay from one CPU generator.
    """
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    inner = n_heads * d_head

    def linear(n_out: int, n_in: int) -> torch.Tensor:
        return torch.randn(n_out, n_in, generator=gen, dtype=torch.float32) * n_in ** -0.5

    p = {f"{n}.weight": linear(inner, d_model) for n in ("q_proj", "k_proj", "v_proj", "g_proj")}
    p["o_proj.weight"] = linear(d_model, inner)
    p["log_decay"] = torch.log(torch.rand(n_heads, generator=gen, dtype=torch.float32) * 0.09 + 0.9)
    return p


def layer_input(B: int, T: int, d_model: int, seed: int = 1):
    """Seeded layer input x and upstream gradient dy, both ``[B, T, d_model]`` fp32 N(0, 1)."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    x = torch.randn(B, T, d_model, generator=gen, dtype=torch.float32)
    dy = torch.randn(B, T, d_model, generator=gen, dtype=torch.float32)
    return x, dy


def sketch_vectors(n_out: int, n_in: int, seed: int):
    """Seeded N(0, 1) probe vectors (r_out [n_out], r_in [n_in]) for a matrix sketch
    ``(W r_in, r_out W)``: two projections that compare a weight gradient without
    storing it."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    return (torch.randn(n_out, generator=gen, dtype=torch.float64),
            torch.randn(n_in, generator=gen, dtype=torch.float64))
