"""Sharding one fixed KDA problem over ranks: geometry, and gloo ranks on CPU.

Each gloo rank runs ``ShardedScan`` with the CPU oracle (forward, and its
autograd for the backward) standing in for the device scan, and the real
exchange (``all_gather_into_tensor``) between ranks.  The assembled result
must equal the unsharded scan: whole-stream shards exactly, streams split in
time between two ranks to float64 rounding.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from simpletrain_b200.sharding import (Piece, ShardedScan, chunk_shard, piece_param, piece_tensor,
                                       shard_bounds, splits_streams, stream_shard)


def test_shard_bounds_cover_and_balance():
    for n in (1, 7, 28, 160, 192):
        for world in (1, 2, 4, 8):
            bounds = [shard_bounds(n, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
            sizes = [e - s for s, e in bounds]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("nstreams,nchunks", [(160, 32), (192, 64), (28, 512), (5, 3), (3, 7), (28, 1)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_chunk_shard_tiles_the_chunk_sequence(nstreams, nchunks, world):
    if nstreams < world:
        with pytest.raises(NotImplementedError):
            chunk_shard(nstreams, nchunks, world, 0)
        return
    seen = []
    sizes = []
    for r in range(world):
        ps = chunk_shard(nstreams, nchunks, world, r)
        sizes.append(sum(p.nstreams * (p.c1 - p.c0) for p in ps))
        for i, p in enumerate(ps):
            assert 0 <= p.c0 < p.c1 <= nchunks and p.s0 < p.s1
            if not p.whole:
                assert p.nstreams == 1
                # a piece that begins mid-stream leads, one that ends mid-stream trails
                assert p.starts or i == 0
                assert p.ends or i == len(ps) - 1
            for s in range(p.s0, p.s1):
                seen += [(s, c) for c in range(p.c0, p.c1)]
    assert seen == [(s, c) for s in range(nstreams) for c in range(nchunks)]
    assert max(sizes) - min(sizes) <= 1
    divisible = nstreams % world == 0
    assert splits_streams(nstreams, nchunks, world) == (not divisible and nchunks > 1)


@pytest.mark.parametrize("nstreams,nchunks", [(160, 32), (28, 512), (5, 3), (3, 7)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_stream_shard_gives_whole_streams(nstreams, nchunks, world):
    if nstreams < world:
        with pytest.raises(NotImplementedError):
            stream_shard(nstreams, nchunks, world, 0)
        return
    per = []
    for r in range(world):
        ps = stream_shard(nstreams, nchunks, world, r)
        assert len(ps) == 1 and ps[0].whole
        per.append((ps[0].s0, ps[0].s1))
    assert per[0][0] == 0 and per[-1][1] == nstreams
    assert all(a[1] == b[0] for a, b in zip(per, per[1:]))
    assert max(b - a for a, b in per) - min(b - a for a, b in per) <= 1
    sc = ShardedScan(1, nstreams, nchunks * 64, 8, 64, world, 0, fwd=lambda *a: None, bwd=lambda *a: None)
    assert not sc.split and sc.pieces == stream_shard(nstreams, nchunks, world, 0)
    with pytest.raises(ValueError):
        ShardedScan(1, nstreams, 64, 8, 64, world, 0, fwd=lambda *a: None, bwd=lambda *a: None, balance="x")


def test_the_10b_shape_over_8_ranks_splits_four_heads_in_half():
    split = [p for r in range(8) for p in chunk_shard(28, 512, 8, r) if not p.whole]
    assert [(p.s0, p.c0, p.c1) for p in split] == [
        (3, 0, 256), (3, 256, 512), (10, 0, 256), (10, 256, 512),
        (17, 0, 256), (17, 256, 512), (24, 0, 256), (24, 256, 512)]


def test_piece_views_keep_the_layer_memory_order():
    B, H, T, D = 2, 5, 130, 8
    x = torch.randn(B, T, H, D).transpose(1, 2)          # [B, H, T, D] over [B, T, H, D]
    one_row = Piece(6, 9, 0, 3, 3)                       # b = 1, h = 1..3
    v = piece_tensor(x, one_row, T, 64)
    assert v.shape == (1, 3, T, D) and v.data_ptr() == x[1, 1].data_ptr()
    assert v.stride() == x.stride()
    rows = Piece(0, 10, 0, 3, 3)
    assert piece_tensor(x, rows, T, 64).data_ptr() == x.data_ptr()
    across = Piece(3, 7, 0, 3, 3)                        # (0,3) (0,4) (1,0) (1,1): a copy
    c = piece_tensor(x, across, T, 64)
    assert c.shape == (1, 4, T, D) and torch.equal(c[0, 2], x[1, 0])
    tail = Piece(4, 5, 1, 3, 3)
    assert torch.equal(piece_tensor(x, tail, T, 64), x[0:1, 4:5, 64:130])


@pytest.mark.parametrize("shape", [(), (5,), (5, 8), (2, 5, 8), (2, 5, 8, 8)])
def test_piece_param_broadcasts_per_stream_parameters(shape):
    B, H, D = 2, 5, 8
    p = torch.randn(*shape) if shape else torch.tensor(0.5)
    full = p.view(H, 1) if shape == (5,) else p
    full = full.expand(B, H, *(full.shape[2:] if full.dim() > 2 else full.shape[1:] if full.dim() == 2 else
                              ([1] if full.dim() == 1 else [1])))
    for piece in (Piece(6, 9, 0, 3, 3), Piece(0, 10, 0, 3, 3), Piece(3, 7, 0, 3, 3), Piece(4, 5, 1, 3, 3)):
        got = piece_param(p, piece, B, H)
        flat = full.reshape(B * H, *full.shape[2:])
        ref = flat[piece.s0:piece.s1]
        assert torch.equal(got.reshape(ref.shape), ref), (shape, piece)
    assert piece_param(0.9, Piece(0, 1, 0, 1, 1), B, H) == 0.9


# --------------------------------------------------------------------------- #
# gloo ranks running the oracle
# --------------------------------------------------------------------------- #
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_fns(chunk):
    from oracle.kda_oracle import chunk_scan, decay_bhd1

    def dec(decay, q):
        B, H, _, D = q.shape
        return decay_bhd1(decay, B, H, D, dtype=q.dtype)

    def fwd(q, k, v, g, decay, s0):
        return chunk_scan(q, k, v, g, dec(decay, q), chunk, initial_state=s0, compute_dtype=q.dtype)

    def bwd(q, k, v, g, dy, decay, s0, ds_T, need_ddecay, need_ds0):
        leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v, g)]
        dl = decay.detach().clone().requires_grad_(True)
        sl = s0.detach().clone().requires_grad_(True) if s0 is not None else None
        y, S = chunk_scan(*leaves, dec(dl, q), chunk, initial_state=sl, compute_dtype=q.dtype)
        loss = (y * dy).sum() + ((S * ds_T).sum() if ds_T is not None else 0.0)
        wrt = leaves + [dl] + ([sl] if sl is not None else [])
        grads = torch.autograd.grad(loss, wrt, allow_unused=True)
        dd = grads[4] if need_ddecay else None
        d0 = grads[5] if (need_ds0 and sl is not None) else None
        return grads[0], grads[1], grads[2], grads[3], dd, d0

    return fwd, bwd


def _exchange(tile):
    world = dist.get_world_size()
    out = torch.empty((world * tile.shape[0], *tile.shape[1:]), dtype=tile.dtype)
    dist.all_gather_into_tensor(out, tile.contiguous())
    return out.view(world, *tile.shape)


def _problem(B, H, T, D):
    g = torch.Generator().manual_seed(0)
    f = torch.float64
    x = {n: torch.randn(B, T, H, D, generator=g, dtype=f).transpose(1, 2) for n in ("q", "k", "v", "g", "dy")}
    x["decay"] = torch.rand(H, D, generator=g, dtype=f) * 0.2 + 0.8
    x["s0"] = torch.randn(B, H, D, D, generator=g, dtype=f) * 0.1
    dsT = torch.randn(B, H, D, D, generator=g, dtype=f)
    return x, dsT


def _worker(rank, world, port, B, H, T, D, balance, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        x, dsT = _problem(B, H, T, D)
        fwd, bwd = _oracle_fns(64)
        sc = ShardedScan(B, H, T, D, 64, world, rank, fwd=fwd, bwd=bwd, exchange=_exchange, balance=balance)
        loc = sc.load(x)
        outs = sc.forward(loc)
        dfin = [piece_param(dsT, p, B, H) if p.ends else None for p in sc.pieces]
        grads = sc.backward(loc, dfinal_state=dfin)
        merged = [dict(o, **g) for o, g in zip(outs, grads)]
        f = torch.float64
        shapes = {n: ((B, H, T, D), f) for n in ("y", "dq", "dk", "dv", "dg")}
        shapes.update(final_state=((B, H, D, D), f), ds0=((B, H, D, D), f), ddecay=((B, H, D), f))
        res = sc.assemble(merged, shapes, "cpu")
        if rank == 0:
            (yr, Sr), ref = fwd(x["q"], x["k"], x["v"], x["g"], x["decay"], x["s0"]), None
            ref = bwd(x["q"], x["k"], x["v"], x["g"], x["dy"], x["decay"].expand(B, H, D).clone(), x["s0"], dsT,
                      True, True)
            pairs = {"y": yr, "final_state": Sr, "dq": ref[0], "dk": ref[1], "dv": ref[2], "dg": ref[3],
                     "ddecay": ref[4], "ds0": ref[5]}
            errs = {n: (res[n] - r).abs().max().item() / max(r.abs().max().item(), 1e-30)
                    for n, r in pairs.items()}
            q.put((sc.split, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,H,T,world,balance,split", [
    (2, 3, 192, 2, "chunks", False),   # 6 streams over 2 ranks: whole streams, no exchange
    (1, 3, 200, 2, "chunks", True),    # 3 streams of 4 chunks over 2 ranks: one stream split (ragged tail)
    (1, 5, 130, 4, "chunks", True),    # 15 chunks over 4 ranks: a rank with a leading and a trailing split
    (2, 3, 256, 4, "chunks", True),    # pieces that cross batch rows (copied, not viewed)
    (2, 3, 200, 4, "streams", False),  # 6 whole streams over 4 ranks (2, 2, 1, 1), across batch rows
])
def test_gloo_ranks_reassemble_the_unsharded_scan(B, H, T, world, balance, split):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, H, T, 8, balance, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    was_split, errs = q.get(timeout=5)
    assert was_split == split
    bad = {n: e for n, e in errs.items() if not e <= 1e-10}
    assert not bad, errs
