"""The KDA scan of one fixed problem sharded over ranks, one process per GPU.

The ``B * H`` streams (stream index ``s = b * H + h``) are independent, so the
default split (``balance="streams"``, ``stream_shard``) gives each rank a
contiguous run of whole streams, ``floor`` or ``ceil`` of ``B * H / world``
(``shard_bounds``), and the ranks never communicate.  When the stream count
does not divide by the rank count the busiest rank holds one stream more than
the least busy one; on the 10b shape (28 heads over 8 GPUs: four ranks with 4
streams, four with 3) that costs less than splitting streams, because a
rank's step time is dominated by per-launch costs at that size (one B200,
fwd+bwd of 4 streams of 32768 tokens: 0.247 ms, of 3: 0.229 ms; with the
time split below, 3.5 streams per rank over 8 GPUs: 0.587 ms per step).

``balance="chunks"`` balances chunks exactly instead.  Work unit: one chunk
of one stream; each stream has ``NC = ceil(T / C)`` chunks, and the
stream-major sequence of all ``B * H * NC`` chunks is cut into ``world``
contiguous, balanced ranges, one per rank (``shard_bounds``).  A rank's range
splits at stream boundaries into pieces (``chunk_shard``):

* whole streams ``[s0, s1)``;
* at most one leading piece: the end (chunks ``[c0, NC)``) of a stream begun on
  the rank before;
* at most one trailing piece: the start (chunks ``[0, c1)``) of a stream
  finished on the rank after.

When the stream count divides by the rank count every piece is whole and the
ranks never communicate (streams are independent).  Otherwise -- the 10b shape
has 28 heads for 8 GPUs -- a stream is split in time between two neighbouring
ranks and its carried state crosses the split:

* forward: the rank holding the stream's start scans it from the stream's
  initial state; the ranks exchange these exit states (one all_gather of a
  ``D x D`` fp32 tile per rank); the next rank scans the stream's end from it;
* backward: the rank holding the end runs its backward first, from the entry
  state it received; the ranks exchange ``dL/d(entry state)`` (one all_gather);
  the rank holding the start then runs its backward with that as the gradient
  of its exit state.  ``d(decay)`` of a split stream is the sum of the two
  ranks' parts.

This needs at least as many streams as ranks: then every range is at least one
stream long and a stream meets at most two ranks.  The scan and the exchange
are injectable callables, so the same code runs the CUDA ops over NCCL, or a
CPU restatement over ``gloo``, or all ranks emulated in one process.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple, Union

import torch
import torch.distributed as dist

Tensor = torch.Tensor


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of rank's share of n items; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class Piece:
    """Chunks ``[c0, c1)`` of each of the streams ``[s0, s1)`` (``NC`` chunks per stream)."""

    s0: int
    s1: int
    c0: int
    c1: int
    nchunks: int

    @property
    def nstreams(self) -> int:
        return self.s1 - self.s0

    @property
    def starts(self) -> bool:
        """Holds the first chunk of its streams (its entry state is the stream's initial state)."""
        return self.c0 == 0

    @property
    def ends(self) -> bool:
        """Holds the last chunk of its streams (its exit state is the stream's final state)."""
        return self.c1 == self.nchunks

    @property
    def whole(self) -> bool:
        return self.starts and self.ends

    def times(self, T: int, chunk: int) -> Tuple[int, int]:
        """Token range ``[t0, t1)`` of the piece (the last chunk may be ragged)."""
        return self.c0 * chunk, min(T, self.c1 * chunk)


def chunk_shard(nstreams: int, nchunks: int, world: int, rank: int) -> List[Piece]:
    """Rank's pieces of the stream-major chunk sequence, in stream order."""
    if nstreams < world and nchunks > 0 and world > 1:
        raise NotImplementedError(f"{nstreams} streams over {world} ranks: sharding needs at least as many "
                                  "streams as ranks (a stream may then meet at most two ranks)")
    lo, hi = shard_bounds(nstreams * nchunks, world, rank)
    pieces: List[Piece] = []
    while lo < hi:
        s, c0 = divmod(lo, nchunks)
        if c0 == 0 and hi - lo >= nchunks:
            k = (hi - lo) // nchunks
            pieces.append(Piece(s, s + k, 0, nchunks, nchunks))
            lo += k * nchunks
        else:
            c1 = min(nchunks, c0 + (hi - lo))
            pieces.append(Piece(s, s + 1, c0, c1, nchunks))
            lo += c1 - c0
    return pieces


def stream_shard(nstreams: int, nchunks: int, world: int, rank: int) -> List[Piece]:
    """Rank's whole streams ``[s0, s1)`` (sizes differ by at most one), as one piece."""
    if nstreams < world and nchunks > 0 and world > 1:
        raise NotImplementedError(f"{nstreams} streams over {world} ranks: a rank would hold no stream")
    s0, s1 = shard_bounds(nstreams, world, rank)
    return [Piece(s0, s1, 0, nchunks, nchunks)] if s1 > s0 else []


def splits_streams(nstreams: int, nchunks: int, world: int) -> bool:
    """Whether some stream is split in time between two ranks."""
    return any(not p.whole for r in range(world) for p in chunk_shard(nstreams, nchunks, world, r))


def piece_tensor(x: Tensor, piece: Piece, T: int, chunk: int) -> Tensor:
    """The piece's part of a ``[B, H, T, ...]`` tensor, as a ``[b, h, t, ...]`` tensor.

    A view when the piece's streams lie in one batch row or cover whole batch
    rows (its memory order is then the input's, e.g. the KDA layer's
    ``[B, T, H, D]``); otherwise a contiguous copy shaped ``[1, n, t, ...]``.
    """
    H = x.shape[1]
    t0, t1 = piece.times(T, chunk)
    b0, h0 = divmod(piece.s0, H)
    b1, h1 = divmod(piece.s1 - 1, H)
    if b0 == b1:
        return x[b0:b0 + 1, h0:h1 + 1, t0:t1]
    if h0 == 0 and h1 == H - 1:
        return x[b0:b1 + 1, :, t0:t1]
    rows = [x[s // H, s % H, t0:t1] for s in range(piece.s0, piece.s1)]
    return torch.stack(rows).unsqueeze(0)


def piece_param(p: Optional[Union[float, Tensor]], piece: Piece, B: int, H: int) -> Optional[Union[float, Tensor]]:
    """The piece's streams of a per-stream parameter, shaped like ``piece_tensor``'s
    leading ``[b, h]``: a float passes through; a tensor broadcasting to
    ``[B, H, ...]`` (a scalar, ``[H]`` per head, ``[H, D]`` per key channel,
    ``[B, H, D]``, an initial state ``[B, H, D, D]``) is broadcast first."""
    if p is None or not torch.is_tensor(p):
        return p
    t = p
    if t.dim() == 1 and t.shape[0] == H:
        t = t.view(H, 1)
    if t.dim() < 2:
        t = t.reshape(1, 1, *([1] if t.dim() == 0 else t.shape))
    elif t.dim() == 2:
        t = t.unsqueeze(0)
    t = t.expand(B, H, *t.shape[2:])
    b0, h0 = divmod(piece.s0, H)
    b1, h1 = divmod(piece.s1 - 1, H)
    if b0 == b1:
        return t[b0:b0 + 1, h0:h1 + 1]
    if h0 == 0 and h1 == H - 1:
        return t[b0:b1 + 1]
    rows = [t[s // H, s % H] for s in range(piece.s0, piece.s1)]
    return torch.stack(rows).unsqueeze(0)


def place_piece(dst: Tensor, src: Tensor, piece: Piece, T: Optional[int], chunk: int) -> None:
    """Write a piece's result ``src`` into the global, contiguous ``dst``
    (``[B, H, T, ...]`` with ``T`` given, else a per-stream ``[B, H, ...]``)."""
    if not dst.is_contiguous():
        raise ValueError("place_piece writes into a contiguous destination")
    flat = dst.view(-1, *dst.shape[2:])
    rows = src.reshape(piece.nstreams, *src.shape[2:])
    if T is None:
        flat[piece.s0:piece.s1] = rows
    else:
        t0, t1 = piece.times(T, chunk)
        flat[piece.s0:piece.s1, t0:t1] = rows


# --------------------------------------------------------------------------- #
# the sharded scan
# --------------------------------------------------------------------------- #
PER_TOKEN = ("y", "dq", "dk", "dv", "dg")   # results shaped [B, H, T, D]; the rest are per stream

FwdFn = Callable[..., Tuple[Tensor, Tensor]]
BwdFn = Callable[..., Tuple[Tensor, Tensor, Tensor, Optional[Tensor], Optional[Tensor], Optional[Tensor]]]


def cuda_scan_fns(chunk: int = 64, mode: int = 0) -> Tuple[FwdFn, BwdFn]:
    """The ``kda_b200`` ops as the sharded scan's forward and backward."""
    from .ops import decay_as_bhd

    def dec(decay, q):
        B, H, _, D = q.shape
        return decay_as_bhd(decay, B, H, D)

    def fwd(q, k, v, g, decay, s0):
        dt, ds = dec(decay, q)
        return torch.ops.kda_b200.chunk_fwd(q, k, v, g, dt, ds, s0, chunk, mode, True)

    def bwd(q, k, v, g, dy, decay, s0, ds_T, need_ddecay, need_ds0):
        dt, ds = dec(decay, q)
        dq, dk, dv, dg, dd, d0 = torch.ops.kda_b200.chunk_bwd(
            q, k, v, g, dy, dt, ds, s0, None, ds_T, chunk, mode, bool(need_ddecay and dt is not None),
            bool(need_ds0))
        return (dq, dk, dv, dg if g is not None else None,
                dd if dd.numel() else None, d0 if d0.numel() else None)

    return fwd, bwd


def nccl_exchange(group=None) -> Callable[[Tensor], Tensor]:
    """All-gather of one tile per rank: ``[...]`` -> ``[world, ...]``."""

    def exchange(tile: Tensor) -> Tensor:
        world = dist.get_world_size(group)
        out = torch.empty((world * tile.shape[0], *tile.shape[1:]), dtype=tile.dtype, device=tile.device)
        dist.all_gather_into_tensor(out, tile.contiguous(), group=group)
        return out.view(world, *tile.shape)

    return exchange


class ShardedScan:
    """One rank's share of a KDA scan (forward, backward) of a fixed ``[B, H, T, D]`` problem.

    ``load(inputs)`` cuts this rank's pieces out of the global inputs (q, k,
    v, g, dy ``[B, H, T, D]``; decay a float or a per-stream tensor; s0
    ``[B, H, D, D]`` or None).  ``forward(x)`` and ``backward(x)`` run them with
    the exchanges described in the module docstring; each returns one dict per
    piece.  ``fwd``, ``bwd`` and ``exchange`` default to the CUDA ops and NCCL.
    ``balance``: ``"streams"`` (whole streams per rank, no exchange) or
    ``"chunks"`` (exactly balanced chunk ranges, streams split in time).
    The phases are also callable one by one (``forward_local``,
    ``forward_exit``, ``forward_rest``; ``backward_local``, ``backward_entry``,
    ``backward_rest``) for drivers that emulate several ranks in one process.
    """

    def __init__(self, B: int, H: int, T: int, D: int, chunk: int = 64, world: int = 1, rank: int = 0,
                 fwd: Optional[FwdFn] = None, bwd: Optional[BwdFn] = None,
                 exchange: Optional[Callable[[Tensor], Tensor]] = None, mode: int = 0,
                 balance: str = "streams"):
        if balance not in ("streams", "chunks"):
            raise ValueError(f"balance must be 'streams' or 'chunks', not {balance!r}")
        self.B, self.H, self.T, self.D, self.chunk = B, H, T, D, chunk
        self.world, self.rank, self.balance = world, rank, balance
        self.nchunks = (T + chunk - 1) // chunk
        shard = chunk_shard if balance == "chunks" else stream_shard
        self.pieces = shard(B * H, self.nchunks, world, rank) if T > 0 else \
            [Piece(*shard_bounds(B * H, world, rank), 0, 0, 0)]
        self.split = T > 0 and balance == "chunks" and splits_streams(B * H, self.nchunks, world)
        if fwd is None or bwd is None:
            f, b = cuda_scan_fns(chunk, mode)
            fwd, bwd = fwd or f, bwd or b
        self.fwd, self.bwd = fwd, bwd
        self.exchange = exchange
        self._entry: Optional[Tensor] = None

    # ------------------------------------------------------------------ #
    def load(self, inputs: Dict[str, Optional[Union[float, Tensor]]]) -> List[Dict[str, object]]:
        """Per piece: q, k, v, g, dy (``[b, h, t, D]``), decay, s0 (stream-starting pieces only)."""
        out = []
        for p in self.pieces:
            d = {}
            for n in ("q", "k", "v", "g", "dy"):
                t = inputs.get(n)
                d[n] = piece_tensor(t, p, self.T, self.chunk) if t is not None else None
            d["decay"] = piece_param(inputs.get("decay", 0.99), p, self.B, self.H)
            s0 = inputs.get("s0")
            d["s0"] = piece_param(s0, p, self.B, self.H) if (s0 is not None and p.starts) else None
            out.append(d)
        return out

    def _tile(self, x, t: Optional[Tensor]) -> Tensor:
        """One rank's exchange tile: ``t`` as ``[D, D]``, or zeros; fp32 (fp64 for fp64 inputs)."""
        ref = x[0]["q"]
        dt = torch.promote_types(ref.dtype, torch.float32)
        if t is None:
            return torch.zeros(self.D, self.D, dtype=dt, device=ref.device)
        return t.reshape(self.D, self.D).to(dt)

    # ---- forward ------------------------------------------------------ #
    def forward_local(self, x) -> List[Optional[Dict[str, Tensor]]]:
        """Pieces that start their streams: no state from another rank needed."""
        out: List[Optional[Dict[str, Tensor]]] = [None] * len(self.pieces)
        for i, p in enumerate(self.pieces):
            if p.starts:
                d = x[i]
                y, S = self.fwd(d["q"], d["k"], d["v"], d["g"], d["decay"], d["s0"])
                out[i] = {"y": y, "final_state": S}
        return out

    def forward_exit(self, x, out) -> Tensor:
        """This rank's contribution to the forward exchange: the exit state of a
        trailing piece that ends mid-stream, else zeros."""
        if self.pieces and not self.pieces[-1].ends and out[-1] is not None:
            return self._tile(x, out[-1]["final_state"])
        return self._tile(x, None)

    def forward_rest(self, x, out, gathered: Optional[Tensor]) -> List[Dict[str, Tensor]]:
        """The leading piece that begins mid-stream, from the previous rank's exit state."""
        self._entry = None
        if self.pieces and not self.pieces[0].starts:
            self._entry = gathered[self.rank - 1].reshape(1, 1, self.D, self.D).contiguous()
            d = x[0]
            y, S = self.fwd(d["q"], d["k"], d["v"], d["g"], d["decay"], self._entry)
            out[0] = {"y": y, "final_state": S}
        return out

    def forward(self, x) -> List[Dict[str, Tensor]]:
        out = self.forward_local(x)
        gathered = self.exchange(self.forward_exit(x, out)) if self.split else None
        return self.forward_rest(x, out, gathered)

    # ---- backward ----------------------------------------------------- #
    def _bwd(self, i, s0, ds_T, need_ddecay, need_ds0):
        d = self._x[i]
        r = self.bwd(d["q"], d["k"], d["v"], d["g"], d["dy"], d["decay"], s0, ds_T, need_ddecay, need_ds0)
        keys = ("dq", "dk", "dv", "dg", "ddecay", "ds0")
        return {k: t for k, t in zip(keys, r) if t is not None}

    def backward_local(self, x, need_ddecay: bool = True, need_ds0: bool = True,
                       dfinal_state: Optional[Sequence[Optional[Tensor]]] = None):
        """Pieces that end their streams (every gradient they need is at hand).
        ``dfinal_state``: per piece, dL/d(final state) of its streams, or None.
        The leading mid-stream piece's ``ds0`` is dL/d(its entry state)."""
        self._x = x
        self._need = (need_ddecay, need_ds0)
        grads: List[Optional[Dict[str, Tensor]]] = [None] * len(self.pieces)
        for i, p in enumerate(self.pieces):
            if not p.ends:
                continue
            dsT = dfinal_state[i] if dfinal_state is not None else None
            if p.starts:
                grads[i] = self._bwd(i, x[i]["s0"], dsT, need_ddecay, need_ds0 and x[i]["s0"] is not None)
            else:
                grads[i] = self._bwd(i, self._entry, dsT, need_ddecay, True)
        return grads

    def backward_entry(self, x, grads) -> Tensor:
        """This rank's contribution to the backward exchange: dL/d(entry state) of a
        leading piece that begins mid-stream, else zeros."""
        if self.pieces and not self.pieces[0].starts and grads[0] is not None:
            return self._tile(x, grads[0]["ds0"])
        return self._tile(x, None)

    def backward_rest(self, x, grads, gathered: Optional[Tensor]):
        """The trailing piece that ends mid-stream, with the next rank's dL/d(entry)
        as the gradient of its exit state."""
        need_ddecay, need_ds0 = self._need
        if self.pieces and not self.pieces[-1].ends:
            dexit = gathered[self.rank + 1].reshape(1, 1, self.D, self.D).contiguous()
            i = len(self.pieces) - 1
            grads[i] = self._bwd(i, x[i]["s0"], dexit, need_ddecay, need_ds0 and x[i]["s0"] is not None)
        if self.pieces and not self.pieces[0].starts and grads[0] is not None:
            grads[0].pop("ds0", None)     # the gradient of an internal boundary, not of an input
        self._x = None
        return grads

    def backward(self, x, need_ddecay: bool = True, need_ds0: bool = True,
                 dfinal_state: Optional[Sequence[Optional[Tensor]]] = None):
        grads = self.backward_local(x, need_ddecay, need_ds0, dfinal_state)
        gathered = self.exchange(self.backward_entry(x, grads)) if self.split else None
        return self.backward_rest(x, grads, gathered)

    # ---- results on one rank ------------------------------------------ #
    def assemble(self, outs: Sequence[Dict[str, Tensor]], shapes: Dict[str, Tuple[Sequence[int], torch.dtype]],
                 device, group=None, dst: int = 0, reduce: bool = True) -> Dict[str, Tensor]:
        """Sum every rank's piece results into global tensors on rank ``dst``
        (``dist.reduce``: each element comes from one rank, the others add
        zeros; a split stream's ``ddecay`` parts add up).  ``shapes`` gives the
        global shape and dtype per name (``[B, H, T, D]`` for the per-token
        results ``PER_TOKEN``, ``[B, H, ...]`` for per-stream ones).  With
        ``reduce=False`` each rank keeps its own part (zeros elsewhere)."""
        res = {}
        for name, (shape, dtype) in shapes.items():
            g = torch.zeros(tuple(shape), dtype=dtype, device=device)
            per_token = name in PER_TOKEN
            for p, o in zip(self.pieces, outs):
                if o is None or name not in o:
                    continue
                if name == "final_state" and not p.ends:
                    continue
                place_piece(g, o[name], p, self.T if per_token else None, self.chunk)
            if self.world > 1 and reduce:
                dist.reduce(g, dst, op=dist.ReduceOp.SUM, group=group)
            res[name] = g
        return res
