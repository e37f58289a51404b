"""The KDA scan over host-resident tensors, streamed through one B200.

The reference's CPU path takes host tensors and returns host tensors
(``kda_chunked_scan(..., use_triton=False)``, kernels/kda_kernel.py:244-297
and :303-328).  ``HostScan`` gives callers whose q/k/v/g (and dy) live in host
memory the same call on the GPU without paying the PCIe transfers one after
the other: it cuts the batch into slices of whole batch rows and runs every
slice through three CUDA streams -- copy in, scan (forward, and the backward
when ``dy`` is given), copy out -- so the host-to-device copy of slice i+1,
the kernels of slice i and the device-to-host copy of slice i-1 run at the
same time, and the two PCIe directions overlap each other.

Batch rows are independent (b, h) streams of the scan, so a slice needs no
carry from another slice; the decay gradient of a decay shared over the
batch is summed over all rows on the device before it is copied back.

Host tensors should be pinned (``pin_memory=True``): copies from pageable
memory are staged by the driver and overlap nothing.  Device buffers and the
pinned result buffers are kept for the next call with the same shapes; the
returned tensors are those buffers.  ``scan(...)`` returns when its results
are on the host, valid until the second call after it (clone them to keep
them).  ``scan.submit(...)`` returns at once with a ``Pending`` whose
``wait()`` gives the results: two submitted calls overlap (the next call's
copies in run while this one's results come back), with two sets of result
buffers used in turn, so a call's results stay valid until the second
submission after it, which first waits for it.  A submitted call's host
inputs must stay unchanged until its ``wait()`` returns.

``ShardedHostScan`` does the same for one rank's shard of a problem split over
several GPUs (``sharding.ShardedScan``), pipelining whole steps.
"""
from __future__ import annotations

from typing import Dict, Optional, Union

import torch
from torch import Tensor

from .ops import MODE_CORRECTED, MODE_LITERAL, MODE_PER_STEP, decay_as_bhd, per_step_decay

__all__ = ["HostScan", "Pending", "ShardedHostScan"]

_DTYPES = (torch.bfloat16, torch.float16)


def _pinned_like(t: Tensor) -> Tensor:
    return torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device="cpu", pin_memory=True)


class Pending:
    """A submitted ``HostScan`` call: ``wait()`` blocks until its results are on the host."""

    def __init__(self, results: Dict[str, Tensor], finished: torch.cuda.Event):
        self._results = results
        self._finished = finished

    def wait(self) -> Dict[str, Tensor]:
        self._finished.synchronize()
        return self._results


class HostScan:
    """KDA chunked scan (forward, optionally backward) of host tensors on one GPU.

    ``HostScan(device=None, slices=None, chunk_size=64, per_step=False,
    reference_exact=False)``; ``slices`` defaults to ``min(B, 16)`` batch
    slices (on the 1b shape, B=16, fwd+bwd, one call at a time: 4 slices
    2.68 M, 8 slices 2.84 M, 16 slices 2.96 M tokens/s; with ``submit``
    overlapping consecutive calls, 3.1-3.3 M).  Calling it with q, k, v
    (``[B, H, T, D]`` bf16/fp16 host tensors, any strides with the batch
    dimension outermost in memory, such as the ``[B, T, H, D]``-memory views
    the KDA layer produces), an optional gate,
    the decay (float or tensor, as for ``kda_chunk``), an optional ``dy`` and
    initial state returns a dict of host tensors: ``y`` and ``final_state``;
    with ``dy`` also ``dq``, ``dk``, ``dv``, ``dg`` (with a gate), ``ddecay``
    (a tensor decay, not per-step) and ``ds0`` (with an initial state) -- the
    gradients of ``sum(y * dy)``.
    """

    def __init__(self, device: Optional[Union[int, str, torch.device]] = None, slices: Optional[int] = None,
                 chunk_size: int = 64, per_step: bool = False, reference_exact: bool = False):
        if per_step and reference_exact:
            raise ValueError("per_step and reference_exact are different semantics; pick one")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("HostScan streams host tensors through a CUDA device")
        self.slices = slices
        self.chunk = int(chunk_size)
        self.mode = MODE_PER_STEP if per_step else (MODE_LITERAL if reference_exact else MODE_CORRECTED)
        self.per_step = per_step
        self._key = None
        self._streams = None
        self._pending = [None, None]   # the last call on each result-buffer set
        self._turn = 0                 # result-buffer set of the next call
        self._slice_done = []          # per slice: the last call's scan of it (reads the device inputs)

    # ------------------------------------------------------------------ #
    def _buffers(self, key, tensors: Dict[str, Tensor], outs: Dict[str, tuple]):
        """(Re)allocate device inputs and two sets of pinned host results for a new shape."""
        if key == self._key:
            return
        for p in self._pending:   # calls in flight still use the old buffers
            if p is not None:
                p.wait()
        self._pending = [None, None]
        self._slice_done = []
        self.dev_in = {n: torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device=self.device)
                       for n, t in tensors.items()}
        self.host_out = []
        for _ in range(2):
            ho = {}
            for n, (like, shape) in outs.items():
                if like is not None:
                    ho[n] = _pinned_like(like)
                else:
                    ho[n] = torch.empty(shape, dtype=torch.float32, pin_memory=True)
            self.host_out.append(ho)
        self._key = key

    def __call__(self, q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor] = None,
                 decay: Union[float, Tensor] = 0.99, dy: Optional[Tensor] = None,
                 initial_state: Optional[Tensor] = None, output_final_state: bool = True) -> Dict[str, Tensor]:
        return self.submit(q, k, v, g, decay, dy, initial_state, output_final_state).wait()

    def submit(self, q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor] = None,
               decay: Union[float, Tensor] = 0.99, dy: Optional[Tensor] = None,
               initial_state: Optional[Tensor] = None, output_final_state: bool = True) -> Pending:
        """Queue the call and return at once; ``wait()`` on the result gives what ``__call__`` returns."""
        if q.dim() != 4:
            raise ValueError(f"q must be [B, H, T, D], got shape {tuple(q.shape)}")
        if q.dtype not in _DTYPES:
            raise TypeError(f"KDA sm_100a kernels take bf16/fp16 inputs, got {q.dtype}")
        B, H, T, D = q.shape
        named = {"q": q, "k": k, "v": v}
        if g is not None:
            named["g"] = g
        if dy is not None:
            named["dy"] = dy
        for n, t in named.items():
            if t.device.type != "cpu":
                raise ValueError(f"HostScan takes host tensors; {n} is on {t.device}")
            if t.shape != q.shape or t.dtype != q.dtype:
                raise ValueError(f"{n} must match q's shape {tuple(q.shape)} and dtype {q.dtype}")
            if t.stride(0) != max(t.stride()) and B > 1:
                raise ValueError(f"{n}: the batch dimension must be outermost in memory")
        if initial_state is not None:
            if initial_state.shape != (B, H, D, D) or initial_state.device.type != "cpu":
                raise ValueError(f"initial_state must be a host [B, H, D, D] = {(B, H, D, D)} tensor")
            named["s0"] = initial_state.float()
        backward = dy is not None
        dec_t = decay if torch.is_tensor(decay) else None
        want_dd = backward and dec_t is not None and not self.per_step
        want_ds0 = backward and initial_state is not None

        outs = {"y": (q, None)}
        if output_final_state:
            outs["final_state"] = (None, (B, H, D, D))
        if backward:
            outs.update(dq=(q, None), dk=(q, None), dv=(q, None))
            if g is not None:
                outs["dg"] = (q, None)
            if want_dd:
                outs["ddecay"] = (None, tuple(dec_t.shape))
            if want_ds0:
                outs["ds0"] = (None, (B, H, D, D))
        key = (tuple(q.shape), q.dtype, tuple((n, t.stride()) for n, t in named.items()),
               tuple(outs), None if dec_t is None else tuple(dec_t.shape))
        self._buffers(key, named, outs)  # outside inference mode: the results are ordinary tensors
        with torch.inference_mode():  # the ops are called directly: no autograd layer per call
            return self._run(named, q, g, decay, dec_t, backward, want_dd, want_ds0, output_final_state)

    def _run(self, named, q, g, decay, dec_t, backward, want_dd, want_ds0, output_final_state):
        B, H, T, D = q.shape
        dev = self.device
        if self._streams is None:
            self._streams = [torch.cuda.Stream(device=dev) for _ in range(3)]
        s_in, s_run, s_out = self._streams
        caller = torch.cuda.current_stream(dev)

        # the decay, whole, on the device first (small); its [B, H, D] view is sliced per slice
        with torch.cuda.stream(s_run):
            s_run.wait_stream(caller)
            dd = dec_t.to(dev, non_blocking=True) if dec_t is not None else decay
            if self.per_step:
                dview, dscal = per_step_decay(dd, B, H, D, q.dtype)
            else:
                dview, dscal = decay_as_bhd(dd, B, H, D)
            dd_rows = torch.empty((B, H, D), dtype=torch.float32, device=dev) if want_dd else None
        s_in.wait_stream(caller)

        # this call's result buffers: the set of the call before the last, once that has finished
        turn = self._turn
        self._turn ^= 1
        if self._pending[turn] is not None:
            self._pending[turn].wait()
        n_sl = max(1, min(B, self.slices if self.slices is not None else 16))
        bounds = [(B * i // n_sl, B * (i + 1) // n_sl) for i in range(n_sl)]
        di, ho = self.dev_in, self.host_out[turn]
        prev_done, slice_done = self._slice_done, []
        for i, (b0, b1) in enumerate(bounds):
            if b1 == b0:
                continue
            # copy in, once the last call's scan of this slice has read the device inputs
            with torch.cuda.stream(s_in):
                if i < len(prev_done) and prev_done[i] is not None:
                    s_in.wait_event(prev_done[i])
                for n, t in named.items():
                    di[n][b0:b1].copy_(t[b0:b1], non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(s_in)
            # scan
            with torch.cuda.stream(s_run):
                s_run.wait_event(arrived)
                sl = {n: t[b0:b1] for n, t in di.items()}
                dv_sl = dview[b0:b1] if dview is not None else None
                s0 = sl.get("s0")
                y, sT = torch.ops.kda_b200.chunk_fwd(sl["q"], sl["k"], sl["v"], sl.get("g"), dv_sl, dscal, s0,
                                                      self.chunk, self.mode, bool(output_final_state))
                res = {"y": y}
                if output_final_state:
                    res["final_state"] = sT
                if backward:
                    gq, gk, gv, gg, gd, gs0 = torch.ops.kda_b200.chunk_bwd(
                        sl["q"], sl["k"], sl["v"], sl.get("g"), sl["dy"], dv_sl, dscal, s0, None, None,
                        self.chunk, self.mode, want_dd, want_ds0)
                    res.update(dq=gq, dk=gk, dv=gv)
                    if g is not None:
                        res["dg"] = gg
                    if want_dd:
                        dd_rows[b0:b1].copy_(gd)
                    if want_ds0:
                        res["ds0"] = gs0
                done = torch.cuda.Event()
                done.record(s_run)
            while len(slice_done) < i:
                slice_done.append(None)
            slice_done.append(done)
            # copy out
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for n, t in res.items():
                    t.record_stream(s_out)
                    ho[n][b0:b1].copy_(t, non_blocking=True)
        if want_dd:
            with torch.cuda.stream(s_run):
                # d(decay) of the broadcast decay: summed over the rows it was broadcast to
                d = dec_t.reshape(H, 1) if dec_t.dim() == 1 and dec_t.shape[0] == H else dec_t
                red = dd_rows.sum_to_size(d.shape).reshape(dec_t.shape)
                done = torch.cuda.Event()
                done.record(s_run)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                red.record_stream(s_out)
                ho["ddecay"].copy_(red, non_blocking=True)
        self._slice_done = slice_done
        finished = torch.cuda.Event()
        finished.record(s_out)
        pending = Pending(dict(ho), finished)
        self._pending[turn] = pending
        return pending


class ShardedHostScan:
    """One rank's shard of a sharded scan (``sharding.ShardedScan``), fed from
    and returned to host memory, with consecutive steps pipelined.

    ``submit(pieces)`` takes this rank's pieces as host tensors -- the dicts
    ``ShardedScan.load`` makes, from pinned host inputs -- copies them to the
    device on a copy-in stream, runs the forward (and the backward when the
    pieces carry ``dy``) with the scan's exchanges on a compute stream, and
    copies every result back to pinned host buffers on a copy-out stream.  It
    returns with a ``Pending``; device inputs and host results come in
    ``sets`` sets (default 2) used in turn, so step i+1's copies in run while
    step i computes and step i-1's results come back, and the two PCIe
    directions overlap.  A submission queues its copies in and its scan at
    once and waits on the host only before queueing its copies out, for the
    call that last used its set.  Results: per piece a dict with ``y``,
    ``final_state`` and, with ``dy``, ``dq``, ``dk``, ``dv``, ``dg``,
    ``ddecay`` (a tensor decay), ``ds0`` (a piece that holds the stream's
    initial state).  A call's results stay valid until the ``sets``-th
    submission after it, which first waits for it: with three sets a caller
    can read step i-2's results after submitting step i and keep both copy
    directions busy.  All ranks must submit the same number of steps (the
    exchanges are collectives).
    """

    def __init__(self, scan, device: Optional[Union[int, str, torch.device]] = None,
                 need_ddecay: bool = True, need_ds0: bool = True, sets: int = 2):
        if sets < 2:
            raise ValueError("ShardedHostScan needs at least two buffer sets")
        self.scan = scan
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.need = (need_ddecay, need_ds0)
        self._streams = [torch.cuda.Stream(device=self.device) for _ in range(3)]
        self._dev = [None] * sets      # device inputs per buffer set
        self._host = [None] * sets     # pinned host results per buffer set
        self._busy = [None] * sets     # per set: the event after which its device inputs are free
        self._pending = [None] * sets
        self._turn = 0

    @staticmethod
    def _to_device_like(piece, dev):
        out = {}
        for n, t in piece.items():
            out[n] = (torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device=dev)
                      if torch.is_tensor(t) else t)
        return out

    def submit(self, pieces) -> Pending:
        s_in, s_run, s_out = self._streams
        caller = torch.cuda.current_stream(self.device)
        turn = self._turn
        self._turn = (turn + 1) % len(self._dev)
        if self._dev[turn] is None:
            self._dev[turn] = [self._to_device_like(p, self.device) for p in pieces]
        dev = self._dev[turn]
        # Copies in and the scan are queued before the host waits for anything: they depend
        # only on device work (the scan that last read these device buffers), so the copy-in
        # stream never runs dry while the host waits; only the copies out, which overwrite
        # the result buffers of the call two submissions back, are queued after that wait.
        with torch.cuda.stream(s_in):
            s_in.wait_stream(caller)
            if self._busy[turn] is not None:
                s_in.wait_event(self._busy[turn])
            for hp, dp in zip(pieces, dev):
                for n, t in hp.items():
                    if torch.is_tensor(t):
                        dp[n].copy_(t, non_blocking=True)
            arrived = torch.cuda.Event()
            arrived.record(s_in)
        with torch.cuda.stream(s_run), torch.inference_mode():
            s_run.wait_event(arrived)
            outs = self.scan.forward(dev)
            if dev and dev[0].get("dy") is not None:
                grads = self.scan.backward(dev, *self.need)
                outs = [dict(o, **g) for o, g in zip(outs, grads)]
            outs = [{n: t for n, t in o.items() if not (n == "final_state" and not p.ends)}
                    for o, p in zip(outs, self.scan.pieces)]
            done = torch.cuda.Event()
            done.record(s_run)
        self._busy[turn] = done
        if self._pending[turn] is not None:
            self._pending[turn].wait()
        if self._host[turn] is None:
            self._host[turn] = [{n: torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for n, t in o.items()}
                                for o in outs]
        host = self._host[turn]
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for o, ho in zip(outs, host):
                for n, t in o.items():
                    t.record_stream(s_out)
                    ho[n].copy_(t, non_blocking=True)
            finished = torch.cuda.Event()
            finished.record(s_out)
        pend = Pending(host, finished)
        self._pending[turn] = pend
        return pend

    @staticmethod
    def nbytes(pieces) -> int:
        """Bytes of the tensors in a list of piece dicts (inputs or results)."""
        return sum(t.numel() * t.element_size() for p in pieces for t in p.values() if torch.is_tensor(t))
