"""torch ops over the sm_100a KDA C ABI, with autograd.

``kda_b200::chunk_fwd`` and ``kda_b200::chunk_bwd`` are defined and
implemented in C++ (``csrc/torch_ops.cpp``, built into
``_lib/kda_b200_ops.so``): they call ``kda_fwd_sm100`` / ``kda_bwd_sm100``
(``include/kda_sm100.h``) on torch's current CUDA stream, with outputs and
workspace from the caching allocator, so they can be captured in CUDA graphs.
This module loads them and registers their fake implementations (for
``torch.compile`` tracing) and the autograd formula.  A nonzero ABI status
raises ``RuntimeError``.  There is no CPU or fallback path: CPU tensors are
rejected, and a missing build raises ``ImportError``.
"""
from __future__ import annotations

import os
from typing import Optional, Tuple, Union

import torch

from . import _ffi

TORCH_OPS = os.path.join(_ffi.LIB_DIR, "kda_b200_ops.so")

Tensor = torch.Tensor

_DTYPES = {torch.bfloat16: _ffi.KDA_DTYPE_BF16, torch.float16: _ffi.KDA_DTYPE_F16}

if not os.path.exists(TORCH_OPS):
    raise ImportError(f"KDA torch ops not built ({TORCH_OPS}); run `python -m simpletrain_b200.build`")
_ffi.load()                       # the C ABI library (status strings, diagnostics)
torch.ops.load_library(TORCH_OPS)  # defines kda_b200::chunk_fwd / chunk_bwd / status_word


def _lib():
    return _ffi.load()


def status_word(device: torch.device) -> Tensor:
    """Per-device int32 word the kernels OR device-side error bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch.ops.kda_b200.status_word(idx)


def device_status(device: Union[torch.device, int, None] = None, reset: bool = True) -> int:
    """Read (and by default clear) the device-side error bits.  Synchronises."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    w = status_word(device)
    val = int(w.item())
    if reset and val:
        w.zero_()
    return val


def _abi_layout_ok(t: Tensor) -> bool:
    if t.stride(-1) != 1 and t.shape[-1] != 1:
        return False
    if t.data_ptr() % 16:
        return False
    return all(s % 8 == 0 for n, s in zip(t.shape[:-1], t.stride()[:-1]) if n != 1)


def _prep(t: Optional[Tensor]) -> Optional[Tensor]:
    if t is None:
        return None
    return t if _abi_layout_ok(t) else t.contiguous()


def _desc(t: Optional[Tensor]) -> _ffi.KdaTensor:
    if t is None:
        return _ffi.KdaTensor(None, 0, 0, 0, 0)
    st = [0 if n == 1 else s for n, s in zip(t.shape, t.stride())]
    st[3] = 1
    return _ffi.KdaTensor(t.data_ptr(), *st)


def _ptr(t: Optional[Tensor]):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _decay_fields(decay: Optional[Tensor]):
    if decay is None:
        return None, 0, 0, 0
    st = [0 if n == 1 else s for n, s in zip(decay.shape, decay.stride())]
    return decay.data_ptr(), st[0], st[1], st[2]


def _validate(q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor], chunk: int):
    if q.device.type != "cuda":
        raise RuntimeError("the KDA sm_100a kernels need CUDA tensors (there is no CPU path)")
    if q.dim() != 4:
        raise ValueError(f"q must be [B, H, T, D], got shape {tuple(q.shape)}")
    for n, t in (("k", k), ("v", v), ("gate", g)):
        if t is None:
            continue
        if t.shape != q.shape:
            raise ValueError(f"{n} shape {tuple(t.shape)} != q shape {tuple(q.shape)}")
        if t.dtype != q.dtype or t.device != q.device:
            raise TypeError(f"{n} must match q's dtype and device")
    if q.dtype not in _DTYPES:
        raise TypeError(f"KDA sm_100a kernels take bf16/fp16 inputs, got {q.dtype}")


# --------------------------------------------------------------------------- #
# fake implementations (shapes only) for tracing
# --------------------------------------------------------------------------- #
# state-update semantics passed to the ops
MODE_CORRECTED, MODE_LITERAL, MODE_PER_STEP = 0, 1, 2


@torch.library.register_fake("kda_b200::chunk_fwd")
def _(q, k, v, g, decay, decay_scalar, s0, chunk, mode, want_state):
    B, H, T, D = q.shape
    shape = (B, H, D, D) if want_state else (0,)
    return torch.empty_like(q), q.new_empty(shape, dtype=torch.float32)


@torch.library.register_fake("kda_b200::chunk_bwd")
def _(q, k, v, g, dy, decay, decay_scalar, s0, s_T, ds_T, chunk, mode, need_ddecay, need_ds0):
    B, H, T, D = q.shape
    f32 = torch.float32
    dg = torch.empty_like(g) if g is not None else q.new_empty((0,))
    dd = q.new_empty((B, H, D) if (need_ddecay and decay is not None) else (0,), dtype=f32)
    ds0 = q.new_empty((B, H, D, D) if need_ds0 else (0,), dtype=f32)
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), dg, dd, ds0


# --------------------------------------------------------------------------- #
# autograd
# --------------------------------------------------------------------------- #
def _setup_context(ctx, inputs, output):
    q, k, v, g, decay, decay_scalar, s0, chunk, mode, want_state = inputs
    y, s_T = output
    ctx.save_for_backward(q, k, v, g, decay, s0, s_T if want_state else None)
    ctx.decay_scalar = decay_scalar
    ctx.chunk = chunk
    ctx.mode = mode
    ctx.has_gate = g is not None


def _backward(ctx, dy, ds_T):
    q, k, v, g, decay, s0, s_T = ctx.saved_tensors
    need = ctx.needs_input_grad
    need_ddecay = bool(need[4]) and decay is not None
    if need_ddecay and ctx.mode == MODE_PER_STEP:
        raise NotImplementedError("per-step mode does not differentiate the decay")
    need_ds0 = bool(need[6]) and s0 is not None
    if dy is None:
        dy = torch.zeros_like(q)
    use_dsT = ds_T is not None and ds_T.numel() > 0 and s_T is not None
    dq, dk, dv, dg, ddecay, ds0 = torch.ops.kda_b200.chunk_bwd(
        q, k, v, g, dy, decay, ctx.decay_scalar, s0,
        s_T if use_dsT else None, ds_T if use_dsT else None,
        ctx.chunk, ctx.mode, need_ddecay, need_ds0)
    return (dq, dk, dv, dg if ctx.has_gate else None,
            ddecay if need_ddecay else None, None,
            ds0 if need_ds0 else None, None, None, None)


torch.library.register_autograd("kda_b200::chunk_fwd", _backward, setup_context=_setup_context)


# --------------------------------------------------------------------------- #
# extended public API
# --------------------------------------------------------------------------- #
def decay_as_bhd(decay: Union[float, Tensor], B: int, H: int, D: int) -> Tuple[Optional[Tensor], float]:
    """Normalise the extended API's decay to (fp32 [B,H,D] view or None, scalar).

    Accepted: a Python float; a tensor of shape (), (H,) (per head), (H, D)
    (per key channel), (B, H, D), or anything broadcastable to (B, H, D).
    """
    if not torch.is_tensor(decay):
        return None, float(decay)
    d = decay.float()
    if d.dim() == 1 and d.shape[0] == H:
        d = d.view(H, 1)
    return torch.broadcast_to(d, (B, H, D)), 0.0


def per_step_decay(decay: Union[float, Tensor], B: int, H: int, D: int,
                   dtype: torch.dtype = torch.bfloat16) -> Tuple[Optional[Tensor], float]:
    """Per-step decay as (fp32 [B,H,D] view constant along D, or None, scalar).

    Accepted: a float in [0.125, 1] (fp16 inputs: [0.9, 1], the powers
    a^-32 .. a^32 the kernels scale q and k rows by must fit fp16), or a tensor
    of shape (), (H,) (per head) or anything broadcastable to (B, H, 1) (one
    decay per batch and head) with values in the same range.
    """
    if not torch.is_tensor(decay):
        a = float(decay)
        lo = 0.9 if dtype == torch.float16 else 0.125
        if not lo <= a <= 1.0:
            raise ValueError(f"per-step decay must lie in [{lo}, 1] for {dtype}, got {a}")
        return None, a
    if decay.requires_grad:
        raise NotImplementedError("per-step mode does not differentiate the decay")
    d = decay.float()
    if d.dim() == 1 and d.shape[0] == H:
        d = d.view(H, 1)
    if d.dim() >= 1 and d.shape[-1] != 1:
        raise ValueError("per-step decay is one value per (batch, head): its last dimension must be 1")
    return torch.broadcast_to(d, (B, H, 1)).expand(B, H, D), 0.0


def kda_chunk(q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor] = None,
              decay: Union[float, Tensor] = 0.99, initial_state: Optional[Tensor] = None,
              chunk_size: int = 64, reference_exact: bool = False,
              output_final_state: bool = True, per_step: bool = False) -> Tuple[Tensor, Optional[Tensor]]:
    """KDA chunked scan on B200: returns ``(y, final_state)``.

    q, k, v, g: ``[B, H, T, D]`` bf16/fp16 CUDA tensors (any strides; the
    ``[B, T, H, D]``-memory views the KDA layer produces are used in place).
    decay: float or tensor (see ``decay_as_bhd``); per chunk of length L the
    state's key-channel rows are scaled by ``decay**L``.  initial_state:
    ``[B, H, D, D]`` fp32 or None (zeros).  ``reference_exact`` selects the
    reference's literal ``K V^T`` state update (``kernels/kda_kernel.py:294``,
    needs D == chunk_size); the default is the ``K^T V`` form.  Differentiable
    in q, k, v, g, a tensor decay and the initial state.

    ``per_step`` selects the per-token recurrence of the reference's docstring
    (``kernels/kda_kernel.py:8-11``): ``s_t = a s_{t-1} + k_t^T v_t``,
    ``y_t = g_t * (q_t s_t)``, with one decay per (batch, head) (see
    ``per_step_decay``); the final state is ``s_T``.  Differentiable in q, k, v,
    g and the initial state (not the decay).
    """
    _validate(q, k, v, g, chunk_size)
    B, H, T, D = q.shape
    if per_step and reference_exact:
        raise ValueError("per_step and reference_exact are different semantics; pick one")
    if reference_exact and D != chunk_size:
        raise RuntimeError(
            f"The size of tensor a ({D}) must match the size of tensor b ({chunk_size}) "
            f"at non-singleton dimension 3")
    if reference_exact and output_final_state and T % chunk_size:
        raise ValueError("reference_exact: the final state of a ragged last chunk is not defined")
    dt, ds = per_step_decay(decay, B, H, D, q.dtype) if per_step else decay_as_bhd(decay, B, H, D)
    if initial_state is not None and initial_state.shape != (B, H, D, D):
        raise ValueError(f"initial_state must be [B, H, D, D] = {(B, H, D, D)}")
    mode = MODE_PER_STEP if per_step else (MODE_LITERAL if reference_exact else MODE_CORRECTED)
    y, s = torch.ops.kda_b200.chunk_fwd(q, k, v, g, dt, ds, initial_state, int(chunk_size),
                                        mode, bool(output_final_state))
    return y, (s if output_final_state else None)
