"""(batch, head) sharding over ranks: world-size-2 gloo ranks on CPU.

Each rank scans its share of the streams (with the CPU oracle standing in for
the device scan, which is per-stream just the same) and the shards are
gathered; the result must equal the unsharded scan exactly.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from simpletrain_b200.sharding import (concat_sizes, gather_streams, shard_bounds, shard_per_stream,
                                       take_streams, unflatten_streams)


def test_shard_bounds_cover_and_balance():
    for n in (1, 7, 28, 160, 192):
        for world in (1, 2, 4, 8):
            bounds = [shard_bounds(n, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
            sizes = concat_sizes(n, world)
            assert max(sizes) - min(sizes) <= 1
    assert concat_sizes(28, 8) == [4, 4, 4, 4, 3, 3, 3, 3]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, H, T, D, q):
    from oracle.kda_oracle import chunk_scan, decay_bhd1
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        x = {n: torch.randn(B, H, T, D, generator=g) for n in ("q", "k", "v", "g")}
        decay = torch.rand(H, D, generator=g) * 0.2 + 0.8
        s0 = torch.randn(B, H, D, D, generator=g) * 0.1
        lo, hi = shard_bounds(B * H, world, rank)
        loc = {n: take_streams(t, lo, hi) for n, t in x.items()}
        dec = shard_per_stream(decay, B, H, lo, hi).unsqueeze(-1)
        s0l = shard_per_stream(s0, B, H, lo, hi)
        y, S = chunk_scan(loc["q"], loc["k"], loc["v"], loc["g"], dec, 64, initial_state=s0l)
        yg = unflatten_streams(gather_streams(y, B * H, world), B, H)
        Sg = unflatten_streams(gather_streams(S, B * H, world), B, H)
        if rank == 0:
            yr, Sr = chunk_scan(x["q"], x["k"], x["v"], x["g"], decay_bhd1(decay, B, H, D), 64, initial_state=s0)
            q.put((torch.equal(yg, yr), torch.equal(Sg, Sr), (yg - yr).abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,H", [(2, 3), (1, 5)])
def test_two_gloo_ranks_reassemble_the_unsharded_scan(B, H):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, H, 96, 8, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    same_y, same_S, err = q.get(timeout=5)
    assert same_y and same_S, err
