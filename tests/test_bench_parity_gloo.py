"""bench.py's multi-rank parity leg on CPU: two gloo ranks hold sharded
outputs of a small call (head-sharded and sequence-sharded layouts), made
by the torch fp32 restatement itself; the leg must accept them and must
reject them when one rank's shard is corrupted."""
import os
import socket
from dataclasses import dataclass

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@dataclass(frozen=True)
class _Wl:
    seq_len: int
    heads: int
    eps: float = 1e-6


def _worker(rank, world, port, mode, corrupt, q_out):
    import sys

    sys.path[:0] = [ROOT, os.path.join(ROOT, "minimax-h3-swift_b200")]
    import torch
    import torch.distributed as dist

    import bench
    from h3attention import BlockList, MaskSpec, torchref
    from h3attention.sharding import head_range, seq_shard_len

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S, H = 1000, 4
        wl = _Wl(S, H)
        bl = BlockList.build(MaskSpec(seq_len=S, frames=10, height=10, width=10, n_random=1, seed=2))
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(S, H, 128, generator=g).to(torch.bfloat16) for _ in range(3))
        wq, wk = (1 + 0.02 * torch.randn(128, generator=g)).to(torch.bfloat16), torch.ones(128).to(torch.bfloat16)
        tab = torch.zeros(S, 64, 4)
        tab[..., 0] = tab[..., 3] = 1.0  # identity rotation
        tab = tab.to(torch.bfloat16)
        qn, kn = torchref.prologue(q, wq, wl.eps, tab), torchref.prologue(k, wk, wl.eps, tab)
        ref = torchref.attend_blocks(qn, kn, v, bl.row_ptr, bl.col_idx, range(bl.n_blocks), range(H), 128 ** -0.5)
        full = torch.zeros(S, H, 128)
        for (h, ib), r in ref.items():
            full[ib * 128:ib * 128 + r.shape[0], h] = r
        full = full.to(torch.bfloat16)
        if mode == "heads":
            h0, h1 = head_range(rank, world, H)
            mine = [t[:, h0:h1].contiguous() for t in (q, k, v, full)]
        else:
            n = seq_shard_len(S, world)

            def shard(t):
                pad = torch.zeros((n * world - S,) + tuple(t.shape[1:]), dtype=t.dtype)
                return torch.cat([t, pad])[rank * n:(rank + 1) * n].contiguous()

            mine = [shard(t) for t in (q, k, v, full)]
        if corrupt and rank == 1:
            mine[3] = (mine[3].float() + 0.5).to(torch.bfloat16)
        res = bench._parity(mode, world, rank, wl, bl, *mine, wq, wk, tab, 128 ** -0.5, torch.device("cpu"))
        if rank == 0:
            q_out.put((res["ok"], res["max_abs"], len(res["per_rank"])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "seq"])
@pytest.mark.parametrize("corrupt", [False, True])
def test_parity_leg_two_ranks(mode, corrupt):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, corrupt, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        ok, max_abs, n = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert n == 2
    assert ok is (not corrupt), (mode, corrupt, max_abs)
