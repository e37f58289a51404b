"""(batch, head) sharding of the KDA scan over ranks, one process per GPU.

Every (batch, head) pair is an independent stream of the scan, so a batch of
streams splits across ranks with no communication on the data path.  A rank
takes a contiguous, balanced range of the flattened B*H streams, runs the scan
on it, and -- only when the caller wants the whole result on one rank, e.g.
to check it -- the shards are gathered with one all_gather per tensor.

The helpers are device-agnostic: with a ``gloo`` group on CPU tensors they
exercise the same index arithmetic as with NCCL on GPUs.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of rank's share of n items; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def take_streams(x: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """Streams [start, end) of a [B, H, ...] tensor, as [1, end-start, ...].

    The flattened stream index is b * H + h.  The result is a view when the
    range stays inside one batch row, a copy otherwise.
    """
    B, H = x.shape[:2]
    flat = x.reshape(B * H, *x.shape[2:]) if x.is_contiguous() else x.flatten(0, 1)
    return flat[start:end].unsqueeze(0)


def gather_streams(local: torch.Tensor, n: int, world: int, group=None) -> torch.Tensor:
    """All-gather per-rank shards [1, n_r, ...] into [n, ...] in stream order."""
    rows = [shard_bounds(n, world, r) for r in range(world)]
    width = max(e - s for s, e in rows)
    x = local.squeeze(0)
    pad = torch.zeros((width, *x.shape[1:]), dtype=x.dtype, device=x.device)
    pad[: x.shape[0]] = x
    parts: List[torch.Tensor] = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[: e - s] for p, (s, e) in zip(parts, rows)], dim=0)


def unflatten_streams(x: torch.Tensor, B: int, H: int) -> torch.Tensor:
    return x.reshape(B, H, *x.shape[1:])


def shard_per_stream(t: torch.Tensor, B: int, H: int, start: int, end: int) -> torch.Tensor:
    """Slice a per-stream parameter (decay [H, D] / [B, H, D], state [B, H, D, D])."""
    if t.dim() >= 2 and t.shape[0] == H and t.dim() in (2,):
        full = t.unsqueeze(0).expand(B, *t.shape)
    else:
        full = t
    return full.reshape(B * H, *full.shape[2:])[start:end].unsqueeze(0)


def rank_workload(B: int, H: int, world: int, rank: int) -> Tuple[int, int]:
    """Convenience: this rank's stream range for a B x H batch."""
    return shard_bounds(B * H, world, rank)


def concat_sizes(n: int, world: int) -> Sequence[int]:
    return [e - s for s, e in (shard_bounds(n, world, r) for r in range(world))]
