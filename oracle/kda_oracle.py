"""CPU oracle for SimpleTrain's KDA chunked scan -- TEST INFRASTRUCTURE ONLY.

This module is test infrastructure, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The CUDA product path never calls it.

What it restates
----------------
SimpleTrain's effective KDA implementation is the pure-PyTorch chunk loop
``_kda_chunked_scan_torch`` (``kernels/kda_kernel.py:244-297``); its Triton
kernel never launches (the wrapper passes an autotuned meta-parameter
explicitly, ``kernels/kda_kernel.py:75-92,232``, and the error is swallowed
into that same torch path at ``:235-238``).  Per chunk of length L
(``:269-275``), with the running fp32 state S (zero-initialised at ``:264``):

    scores  = tril(Q_c K_c^T)                              (:279-280)
    o       = scores V_c + Q_c S                           (:281-287)
    y_c     = (o * g_c).to(y.dtype)   (gate optional)      (:288-290)
    S       = decay**L * S + U_c                           (:293-295)

The reference computes ``U_c = einsum("bhpd,bhqd->bhpq", K_c, V_c)``, i.e.
``K_c V_c^T`` -- an [L, L] time-by-time matrix that only broadcasts into the
[D, D] state when L == D (``:294``).  Two modes are restated here:

* ``literal``   -- exactly that (valid when D == chunk and every chunk that is
                   followed by another one is full); pinned bit-for-bit in
                   spirit against the reference itself by
                   ``tests/golden/make_golden.py``.
* ``corrected`` -- ``U_c = K_c^T V_c`` ([D, D]), the state update the
                   docstrings (``:9``, ``models/kimi_k3.py:67``) and README
                   describe; every shape works.

``decay`` is a Python float (the reference's type, ``:308``) or a tensor that
broadcasts against the ``[B, H, D, D]`` state as ``[B, H, D, 1]`` (per key
channel), which the reference's ``decay ** L * state`` also accepts.

The extensions over the reference (an initial state, the returned final state)
are plain additions to the same loop.  ``manual_backward`` restates, in
float64, the two-direction backward that the CUDA kernels implement, including
the forward-mode decay gradient, so the algorithm itself is checked against
autograd on the CPU.
"""
from __future__ import annotations

from typing import Optional, Tuple, Union

import torch

Decay = Union[float, torch.Tensor]


# --------------------------------------------------------------------------- #
# helpers
# --------------------------------------------------------------------------- #
def max_rel(x: torch.Tensor, ref: torch.Tensor) -> float:
    """Normwise max-relative error: max|x - ref| / max|ref| (0 if ref == 0 and x == ref)."""
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    num = (x - ref).abs().max().item() if x.numel() else 0.0
    den = ref.abs().max().item() if ref.numel() else 0.0
    if den == 0.0:
        return 0.0 if num == 0.0 else float("inf")
    return num / den


def decay_bhd1(decay: Decay, B: int, H: int, D: int, dtype=torch.float32) -> Decay:
    """Map the extended API's decay shapes onto the reference's broadcast form.

    Accepts a float, or a tensor of shape (), (H,), (H, D), (B, H, D) or any
    shape broadcastable to (B, H, D).  Returns a float or a [B, H, D, 1] tensor
    (``kernels/kda_kernel.py:295`` broadcasts it against [B, H, D, D]).
    """
    if not torch.is_tensor(decay):
        return float(decay)
    d = decay.to(dtype)
    if d.dim() == 1 and d.shape[0] == H and H != D:
        d = d.view(H, 1)
    elif d.dim() == 1 and d.shape[0] == H and H == D:
        d = d.view(H, 1)          # (H,) always means per head in the extended API
    return d.expand(B, H, D).unsqueeze(-1)


# --------------------------------------------------------------------------- #
# forward restatement
# --------------------------------------------------------------------------- #
def chunk_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               gate: Optional[torch.Tensor], decay: Decay, chunk_size: int,
               initial_state: Optional[torch.Tensor] = None,
               mode: str = "corrected",
               compute_dtype: torch.dtype = torch.float32) -> Tuple[torch.Tensor, torch.Tensor]:
    """Chunked gated linear attention, returning (y, final_state).

    Follows ``kernels/kda_kernel.py:258-297``: inputs are up-cast to the
    compute dtype (``:259-261``), y is allocated like q (``:263``) and each
    chunk's output is cast back to q's dtype (``:290``).  ``mode`` picks the
    state update (see the module docstring).  Differentiable by autograd.
    """
    if mode not in ("corrected", "literal"):
        raise ValueError(f"mode must be 'corrected' or 'literal', got {mode!r}")
    B, H, T, D = q.shape
    qf, kf, vf = q.to(compute_dtype), k.to(compute_dtype), v.to(compute_dtype)
    gf = gate.to(compute_dtype) if gate is not None else None
    if torch.is_tensor(decay):
        decay = decay.to(compute_dtype)

    y = torch.empty_like(q)
    pieces = []
    if initial_state is None:
        state = torch.zeros(B, H, D, D, dtype=compute_dtype)
    else:
        state = initial_state.to(compute_dtype)
    causal = torch.ones(chunk_size, chunk_size, dtype=compute_dtype).tril()

    for t0 in range(0, T, chunk_size):
        t1 = min(T, t0 + chunk_size)
        L = t1 - t0
        Qc, Kc, Vc = qf[:, :, t0:t1], kf[:, :, t0:t1], vf[:, :, t0:t1]
        scores = torch.matmul(Qc, Kc.transpose(-1, -2)) * causal[:L, :L]
        out = torch.matmul(scores, Vc) + torch.matmul(Qc, state)
        if gf is not None:
            out = out * gf[:, :, t0:t1]
        pieces.append(out.to(y.dtype))
        if mode == "literal":
            update = torch.matmul(Kc, Vc.transpose(-1, -2))      # [L, L]: needs L == D
        else:
            update = torch.matmul(Kc.transpose(-1, -2), Vc)      # [D, D]
        state = (decay ** L) * state + update
    y = torch.cat(pieces, dim=2) if pieces else y
    return y, state


def reference_literal_y(q, k, v, gate, decay, chunk_size):
    """Exactly the reference's output convention: y only, literal update."""
    return chunk_scan(q, k, v, gate, decay, chunk_size, mode="literal")[0]


def naive_recurrence(q, k, v, gate, decay: float, chunk_size: int,
                     initial_state: Optional[torch.Tensor] = None):
    """Per-token restatement of the corrected chunk form (float64, small cases).

    Token t in chunk c sees S_{c-1} (state before its chunk) plus the causal
    sum of k_s v_s^T over s <= t inside the chunk; S_c = a^L S_{c-1} + sum k v.
    Used as an independent known-answer check of ``chunk_scan``.
    """
    B, H, T, D = q.shape
    qd, kd, vd = q.double(), k.double(), v.double()
    gd = gate.double() if gate is not None else None
    S = torch.zeros(B, H, D, D, dtype=torch.float64) if initial_state is None else initial_state.double().clone()
    y = torch.zeros(B, H, T, D, dtype=torch.float64)
    for t0 in range(0, T, chunk_size):
        t1 = min(T, t0 + chunk_size)
        run = torch.zeros_like(S)
        for t in range(t0, t1):
            run = run + kd[:, :, t, :, None] * vd[:, :, t, None, :]
            o = torch.einsum("bhd,bhde->bhe", qd[:, :, t], S + run)
            y[:, :, t] = o * gd[:, :, t] if gd is not None else o
        S = (decay ** (t1 - t0)) * S + run
    return y, S


# --------------------------------------------------------------------------- #
# backward restatement (the algorithm the CUDA kernels implement)
# --------------------------------------------------------------------------- #
def manual_backward(q, k, v, gate, decay_bhd: torch.Tensor, chunk_size: int,
                    initial_state: Optional[torch.Tensor], dy: torch.Tensor,
                    dstate_T: Optional[torch.Tensor] = None, mode: str = "corrected"):
    """Explicit chunk backward in float64 -- the algorithm the CUDA kernels run.

    Gradients of  L = <dy, y> + <dstate_T, S_T>  for y, S_T = chunk_scan(...).
    The forward-direction pass ("A") recomputes S_{c-1} chunk by chunk and
    gives dq, dg and the decay gradient; the reverse pass ("B") carries
    dS_c = dL/dS_c and gives dk, dv and d(initial state).  Neither pass needs
    the other's carry.

    Decay gradient, forward mode: the state's key-channel row i is scaled by
    alpha_c[i] = a[i]**L_c, so its tangent T_c = dS_c/dlog a (row-wise) obeys

        T_c = alpha_c * (T_{c-1} + L_c * S_{c-1}),   T_{-1} = 0,

    and  dL/dlog a[i] = sum_t q_t[i] (dO_t T_{c(t)-1}^T)[i] + <dS_T[i,:], T_T[i,:]>.
    Every term is a product of actual quantities (no large terms cancel), so
    the bf16 tensor-core operands do not limit its accuracy.  Returns
    (dq, dk, dv, dg, d_decay[B,H,D], d_initial_state).
    """
    B, H, T, D = q.shape
    C = chunk_size
    f = torch.float64
    Q, K, V = q.to(f), k.to(f), v.to(f)
    G = gate.to(f) if gate is not None else None
    DY = dy.to(f)
    a = decay_bhd.to(f).reshape(B, H, D)
    S0 = initial_state.to(f) if initial_state is not None else torch.zeros(B, H, D, D, dtype=f)
    causal = torch.ones(C, C, dtype=f).tril()
    chunks = [(t0, min(T, t0 + C)) for t0 in range(0, T, C)]

    def update(Kc, Vc):
        return Kc @ Vc.transpose(-1, -2) if mode == "literal" else Kc.transpose(-1, -2) @ Vc

    dq = torch.zeros_like(Q); dk = torch.zeros_like(K); dv = torch.zeros_like(V)
    dg = torch.zeros_like(Q) if G is not None else None
    dlog = torch.zeros(B, H, D, dtype=f)

    # pass A: forward direction (S and its decay tangent Td)
    S = S0.clone()
    Td = torch.zeros_like(S)
    for (t0, t1) in chunks:
        L = t1 - t0
        Qc, Kc, Vc, DYc = Q[:, :, t0:t1], K[:, :, t0:t1], V[:, :, t0:t1], DY[:, :, t0:t1]
        P = (Qc @ Kc.transpose(-1, -2)) * causal[:L, :L]
        O = P @ Vc + Qc @ S
        if G is not None:
            dg[:, :, t0:t1] = DYc * O
            dO = DYc * G[:, :, t0:t1]
        else:
            dO = DYc
        dP = (dO @ Vc.transpose(-1, -2)) * causal[:L, :L]
        dq[:, :, t0:t1] = dP @ Kc + dO @ S.transpose(-1, -2)
        dlog += (Qc * (dO @ Td.transpose(-1, -2))).sum(dim=2)
        alpha = (a ** L).unsqueeze(-1)
        Td = alpha * (Td + L * S)
        S = alpha * S + update(Kc, Vc)
    if dstate_T is not None:
        dlog += (dstate_T.to(f) * Td).sum(dim=-1)

    # pass B: reverse direction
    dS = dstate_T.to(f).clone() if dstate_T is not None else torch.zeros(B, H, D, D, dtype=f)
    for (t0, t1) in reversed(chunks):
        L = t1 - t0
        Qc, Kc, Vc, DYc = Q[:, :, t0:t1], K[:, :, t0:t1], V[:, :, t0:t1], DY[:, :, t0:t1]
        dO = DYc * G[:, :, t0:t1] if G is not None else DYc
        P = (Qc @ Kc.transpose(-1, -2)) * causal[:L, :L]
        dP = (dO @ Vc.transpose(-1, -2)) * causal[:L, :L]
        if mode == "literal":
            dk_inter = dS @ Vc                     # d/dK of K V^T against dS
            dv_inter = dS.transpose(-1, -2) @ Kc
        else:
            dk_inter = Vc @ dS.transpose(-1, -2)
            dv_inter = Kc @ dS
        dk[:, :, t0:t1] = dP.transpose(-1, -2) @ Qc + dk_inter
        dv[:, :, t0:t1] = P.transpose(-1, -2) @ dO + dv_inter
        dS = Qc.transpose(-1, -2) @ dO + (a ** L).unsqueeze(-1) * dS
    dS0 = dS

    d_decay = torch.where(a != 0, dlog / torch.where(a != 0, a, torch.ones_like(a)), torch.zeros_like(a))
    return dq, dk, dv, dg, d_decay, dS0


# --------------------------------------------------------------------------- #
# per-step (docstring) semantics
# --------------------------------------------------------------------------- #
# The reference's module docstring (kernels/kda_kernel.py:8-11), its README
# (README.md:83-87) and its never-launched Triton kernel (:134-180) describe a
# per-token recurrence instead of the chunk-constant torch loop:
#
#     s_t = a * s_{t-1} + k_t^T v_t,   o_t = q_t s_t,   y_t = g_t * o_t
#
# with one scalar decay a.  (The Triton kernel also multiplies the state by a
# once more after the last token before storing it, :172-189; the final state
# here is s_T, the value the recurrence defines and the one a continuation
# starts from.)
REF_ROW = 32  # reference row of the scaled operands (see per_step_chunk_scan)


def _decay_bh(decay, B: int, H: int) -> torch.Tensor:
    """Per-step decay as a float64 [B, H] tensor (float, (), (H,), or broadcastable to (B, H))."""
    if not torch.is_tensor(decay):
        return torch.full((B, H), float(decay), dtype=torch.float64)
    d = decay.double()
    if d.dim() == 1 and d.shape[0] == H:
        d = d.view(1, H)
    return torch.broadcast_to(d, (B, H)).clone()


def per_step_recurrence(q, k, v, gate, decay, initial_state: Optional[torch.Tensor] = None):
    """The per-token recurrence itself, in float64 (small cases): (y, s_T).

    Differentiable by autograd; the known answer for the per-step kernels.
    """
    B, H, T, D = q.shape
    qd, kd, vd = q.double(), k.double(), v.double()
    gd = gate.double() if gate is not None else None
    a = _decay_bh(decay, B, H)[:, :, None, None]
    S = torch.zeros(B, H, D, D, dtype=torch.float64) if initial_state is None else initial_state.double()
    ys = []
    for t in range(T):
        S = a * S + kd[:, :, t, :, None] * vd[:, :, t, None, :]
        o = torch.einsum("bhd,bhde->bhe", qd[:, :, t], S)
        ys.append(o * gd[:, :, t] if gd is not None else o)
    y = torch.stack(ys, dim=2) if ys else torch.zeros(B, H, 0, D, dtype=torch.float64)
    return y, S


def _row_factors(a: torch.Tensor, n: int, chunk_size: int):
    """fq[b,h,i] = a^(i+1-REF_ROW), fk[b,h,j] = a^(REF_ROW-1-j) for rows 0..n-1."""
    i = torch.arange(n, dtype=torch.float64)
    fq = a[:, :, None] ** (i + 1 - REF_ROW)
    fk = a[:, :, None] ** (REF_ROW - 1 - i)
    return fq, fk


def per_step_chunk_scan(q, k, v, gate, decay, chunk_size: int = 64,
                        initial_state: Optional[torch.Tensor] = None):
    """Chunked form of the per-step recurrence that the sm_100a kernels run (float64).

    Inside a chunk (local rows i, j < L), with m = REF_ROW, only k is scaled,

        K~ = diag(a^(m-1-j)) K                  (so q_i . k~_j = a^(m-1-j) q_i . k_j)
        O  = diag(a^(i+1-m)) [tril(Q K~^T) V + Q (a^m S)]
        S' = a^L S + a^(L-m) K~^T V

    i.e. the chunk-constant kernels' products with a row-scaled k tile, a
    factor per output row and scalar factors on the carried state.  Every
    factor lies in [a^m, a^-m], which is why the kernels take 0.125 <= a <= 1
    (bf16; 0.9 for fp16).
    """
    B, H, T, D = q.shape
    C, m = chunk_size, REF_ROW
    f = torch.float64
    Q, K, V = q.to(f), k.to(f), v.to(f)
    G = gate.to(f) if gate is not None else None
    a = _decay_bh(decay, B, H)
    a4 = a[:, :, None, None]
    S = torch.zeros(B, H, D, D, dtype=f) if initial_state is None else initial_state.to(f).clone()
    fq, fk = _row_factors(a, C, C)
    causal = torch.ones(C, C, dtype=f).tril()
    y = torch.zeros(B, H, T, D, dtype=f)
    for t0 in range(0, T, C):
        t1 = min(T, t0 + C)
        L = t1 - t0
        Qc = Q[:, :, t0:t1]
        Kt = K[:, :, t0:t1] * fk[:, :, :L, None]
        Vc = V[:, :, t0:t1]
        P = (Qc @ Kt.transpose(-1, -2)) * causal[:L, :L]
        O = fq[:, :, :L, None] * (P @ Vc + Qc @ (a4 ** m * S))
        y[:, :, t0:t1] = O * G[:, :, t0:t1] if G is not None else O
        S = a4 ** L * S + a4 ** (L - m) * (Kt.transpose(-1, -2) @ Vc)
    return y, S


def per_step_manual_backward(q, k, v, gate, decay, chunk_size: int,
                             initial_state: Optional[torch.Tensor], dy: torch.Tensor,
                             dstate_T: Optional[torch.Tensor] = None):
    """Explicit backward of ``per_step_chunk_scan`` -- the algorithm of the kernels (float64).

    Gradients of  L = <dy, y> + <dstate_T, s_T>.  With the row factors fq, fk,
    m = REF_ROW and the row-scaled output gradient dO^ = diag(fq) (g * dy)
    (which the forward-direction pass writes for the reverse pass):

      forward direction:  dg = diag(fq) dy * [tril(Q K~^T) V + Q (a^m S_{c-1})]
                          dq = tril(dO^ V^T) K~ + dO^ (a^m S_{c-1})^T
      reverse direction:  dk = diag(fk) [tril(dO^ V^T)^T Q + V (a^(L-m) dS_c)^T]
                          dv = tril(Q K~^T)^T dO^ + K~ (a^(L-m) dS_c)
                          dS_{c-1} = a^L dS_c + a^m Q^T dO^

    Returns (dq, dk, dv, dg, d_initial_state); the decay is not differentiated.
    """
    B, H, T, D = q.shape
    C, m = chunk_size, REF_ROW
    f = torch.float64
    Q, K, V = q.to(f), k.to(f), v.to(f)
    G = gate.to(f) if gate is not None else None
    DY = dy.to(f)
    a = _decay_bh(decay, B, H)
    a4 = a[:, :, None, None]
    S = torch.zeros(B, H, D, D, dtype=f) if initial_state is None else initial_state.to(f).clone()
    fq, fk = _row_factors(a, C, C)
    causal = torch.ones(C, C, dtype=f).tril()
    chunks = [(t0, min(T, t0 + C)) for t0 in range(0, T, C)]
    dq = torch.zeros_like(Q); dk = torch.zeros_like(K); dv = torch.zeros_like(V)
    dg = torch.zeros_like(Q) if G is not None else None

    def tiles(t0, t1):
        L = t1 - t0
        Kt = K[:, :, t0:t1] * fk[:, :, :L, None]
        dO = DY[:, :, t0:t1] * G[:, :, t0:t1] if G is not None else DY[:, :, t0:t1]
        return L, Q[:, :, t0:t1], Kt, V[:, :, t0:t1], fq[:, :, :L, None] * dO

    for (t0, t1) in chunks:
        L, Qc, Kt, Vc, dOh = tiles(t0, t1)
        Sh = a4 ** m * S
        P = (Qc @ Kt.transpose(-1, -2)) * causal[:L, :L]
        if G is not None:
            dg[:, :, t0:t1] = fq[:, :, :L, None] * DY[:, :, t0:t1] * (P @ Vc + Qc @ Sh)
        dP = (dOh @ Vc.transpose(-1, -2)) * causal[:L, :L]
        dq[:, :, t0:t1] = dP @ Kt + dOh @ Sh.transpose(-1, -2)
        S = a4 ** L * S + a4 ** (L - m) * (Kt.transpose(-1, -2) @ Vc)

    dS = dstate_T.to(f).clone() if dstate_T is not None else torch.zeros(B, H, D, D, dtype=f)
    for (t0, t1) in reversed(chunks):
        L, Qc, Kt, Vc, dOh = tiles(t0, t1)
        dSh = a4 ** (L - m) * dS
        P = (Qc @ Kt.transpose(-1, -2)) * causal[:L, :L]
        dP = (dOh @ Vc.transpose(-1, -2)) * causal[:L, :L]
        dk[:, :, t0:t1] = fk[:, :, :L, None] * (dP.transpose(-1, -2) @ Qc + Vc @ dSh.transpose(-1, -2))
        dv[:, :, t0:t1] = P.transpose(-1, -2) @ dOh + Kt @ dSh
        dS = a4 ** L * dS + a4 ** m * (Qc.transpose(-1, -2) @ dOh)
    return dq, dk, dv, dg, dS


# --------------------------------------------------------------------------- #
# the layer around the scan
# --------------------------------------------------------------------------- #
def layer_forward(params: dict, x: torch.Tensor, n_heads: int, d_head: int,
                  chunk_size: int, mode: str) -> torch.Tensor:
    """SimpleTrain's ``KimiDeltaAttention.forward`` (``models/kimi_k3.py:94-125``)
    in fp32 over ``chunk_scan``: [B, T, d_model] -> [B, T, d_model].

    ``params`` holds the layer's tensors by its parameter names (``q_proj.weight``
    ... ``o_proj.weight``, ``log_decay``).  Steps: four bias-free projections
    viewed as [B, H, T, Dh] (``:99-102``); the scan with the detached mean of
    ``exp(log_decay).clamp(1e-3, 0.999)`` as a float decay (``:105-118``); the
    per-head scale by the same clamped exponential, not detached (``:121-122``);
    the transpose back and ``o_proj`` (``:124-125``).  Differentiable by autograd.
    """
    B, T, _ = x.shape
    H, Dh = n_heads, d_head

    def proj(name):
        return torch.matmul(x, params[f"{name}.weight"].t()).view(B, T, H, Dh).transpose(1, 2)

    q, k, v, g = (proj(n) for n in ("q_proj", "k_proj", "v_proj", "g_proj"))
    decay = float(torch.exp(params["log_decay"]).clamp(min=1e-3, max=0.999).detach().mean())
    o, _ = chunk_scan(q, k, v, g, decay, chunk_size, mode=mode)
    head_scale = torch.exp(params["log_decay"]).clamp(min=1e-3, max=0.999)
    o = o * head_scale.view(1, H, 1, 1)
    o = o.transpose(1, 2).contiguous().view(B, T, H * Dh)
    return torch.matmul(o, params["o_proj.weight"].t())
