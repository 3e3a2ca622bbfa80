"""Host logic of the multi-GPU layouts on CPU: world-size-2 gloo process
groups (127.0.0.1), no GPU.  The exchange of the sequence-sharded mode is
checked against the same per-head attention computed unsharded."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from h3attention.sharding import head_range, max_over_ranks, seq_range, seq_shard_len, ulysses_attend


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_range_partitions():
    for heads in (1, 5, 8, 40):
        for world in (1, 2, 3, 4, 8):
            rs = [head_range(r, world, heads) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == heads
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 1


def test_seq_ranges_are_block_aligned_and_cover():
    for S in (1, 128, 4096, 124992, 125632):
        for world in (1, 2, 4, 8):
            n = seq_shard_len(S, world)
            assert n % 128 == 0 and n * world >= S
            rs = [seq_range(r, world, S) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == S
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))


def _dense(q, k, v, seq_len):
    """Per-head softmax attention over the first seq_len tokens, [S, H, D]."""
    qh, kh, vh = (t[:seq_len].transpose(0, 1).double() for t in (q, k, v))
    p = torch.softmax(qh @ kh.transpose(1, 2) / q.shape[-1] ** 0.5, dim=-1)
    out = torch.zeros_like(q, dtype=torch.float64)
    out[:seq_len] = (p @ vh).transpose(0, 1)
    return out.to(q.dtype)


def _worker(rank, world, port, S, H, D, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        n = seq_shard_len(S, world)
        full = [torch.randn(n * world, H, D, generator=g) for _ in range(3)]
        for t in full:
            t[S:] = 0  # padding rows
        mine = [t[rank * n:(rank + 1) * n].clone() for t in full]
        out = ulysses_attend(*mine, seq_len=S, attend=lambda a, b, c: _dense(a, b, c, S))
        want = _dense(*full, S)[rank * n:(rank + 1) * n]
        lo, hi = seq_range(rank, world, S)
        err = (out[: hi - lo] - want[: hi - lo]).abs().max().item() if hi > lo else 0.0
        m = max_over_ranks(float(rank) + 0.5)
        q_out.put((rank, err, tuple(out.shape), m))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S,H", [(300, 4), (1000, 2)])
def test_ulysses_exchange_matches_unsharded(S, H):
    world, D = 2, 16
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, S, H, D, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n = seq_shard_len(S, world)
    for rank, err, shape, m in res:
        assert shape == (n, H, D)
        assert err < 1e-5, (rank, err)
        assert m == world - 0.5



def test_ulysses_rejects_shards_that_do_not_cover_the_sequence():
    with pytest.raises(ValueError):
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
        try:
            x = torch.zeros(128, 3, 8)
            ulysses_attend(x, x, x, seq_len=1000, attend=lambda a, b, c: a)
        finally:
            dist.destroy_process_group()
