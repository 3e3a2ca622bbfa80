"""Sequence-sharded (Ulysses) attention on 2 GPUs over NCCL, against the
single-GPU fused call on the same inputs.  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "minimax-h3-swift_b200")]
    import torch
    import torch.distributed as dist

    from h3attention import BlockList, Runtime
    from h3attention.configs import CONFIGS, EPS
    from h3attention.sharding import cuda_attend_fn, seq_shard_len, ulysses_attend

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        wl = CONFIGS["config1"]
        S, H = wl.seq_len, wl.heads
        rt = Runtime.get(rank)
        n = seq_shard_len(S, world)
        full = [rt.fill_normal(torch.empty((n * world, H, 128), dtype=torch.bfloat16, device=dev), 5, st)
                for st in (1, 2, 3)]
        wq, wk = (rt.fill_normal(torch.empty(128, dtype=torch.bfloat16, device=dev), 5, st, 1.0, 0.02)
                  for st in (4, 5))
        tab = rt.rope_table(torch.from_numpy(wl.positions()).to(dev))
        bl = BlockList.build(wl.mask_spec())
        attend = cuda_attend_fn(rt, bl.on(dev), S, 128 ** -0.5, q_norm=wq, k_norm=wk, eps=EPS, rope_table=tab)
        mine = [t[rank * n:(rank + 1) * n].contiguous() for t in full]
        out = ulysses_attend(*mine, S, attend)
        want = torch.empty_like(full[0])
        rt.attn_fwd(q=full[0][:S], k=full[1][:S], v=full[2][:S], out=want[:S], layout="SHD", scale=128 ** -0.5,
                    blocks=bl.on(dev), q_norm=wq, k_norm=wk, eps=EPS, rope_table=tab)
        torch.cuda.synchronize()
        lo, hi = rank * n, min(S, (rank + 1) * n)
        d = (out[: hi - lo].float() - want[lo:hi].float()).abs()
        q_out.put((rank, d.max().item()))
    finally:
        dist.destroy_process_group()


def test_ulysses_two_gpus_matches_single_gpu(gpu):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err in res:
        assert err == 0.0, (rank, err)  # same kernels, same per-head inputs


def _abi_worker(rank, world, id_q, q_out, chunks=1):
    try:
        _abi_body(rank, world, id_q, q_out, chunks)
    except Exception as e:  # report instead of leaving the parent waiting
        q_out.put((rank, repr(e)))


def _abi_body(rank, world, id_q, q_out, chunks):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "minimax-h3-swift_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["H3C_SEQ_CHUNKS"] = str(chunks)
    import torch

    from h3attention import BlockList, Runtime
    from h3attention.configs import CONFIGS, EPS
    from h3attention.sharding import seq_shard_len

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    wl = CONFIGS["config1"]
    S, H = wl.seq_len, wl.heads
    rt = Runtime.get(rank)
    if rank == 0:  # rank 0 creates the NCCL id and hands it to the others
        uid = Runtime.comm_unique_id()
        for _ in range(world - 1):
            id_q.put(uid)
    else:
        uid = id_q.get(timeout=60)
    n = seq_shard_len(S, world)
    full = [rt.fill_normal(torch.empty((n * world, H, 128), dtype=torch.bfloat16, device=dev), 6, st) for st in (1, 2, 3)]
    wq, wk = (rt.fill_normal(torch.empty(128, dtype=torch.bfloat16, device=dev), 6, st, 1.0, 0.02) for st in (4, 5))
    tab = rt.rope_table(torch.from_numpy(wl.positions()).to(dev))
    bl = BlockList.build(wl.mask_spec())
    rt.comm_init(uid, world, rank)
    mine = [t[rank * n:(rank + 1) * n].contiguous() for t in full]
    out = torch.empty_like(mine[0])
    rt.attn_fwd_seqshard(q=mine[0], k=mine[1], v=mine[2], out=out, layout="SHD", scale=128 ** -0.5,
                         blocks=bl.on(dev), q_norm=wq, k_norm=wk, eps=EPS, rope_table=tab, seq_len=S)
    want = torch.empty_like(full[0])
    rt.attn_fwd(q=full[0][:S], k=full[1][:S], v=full[2][:S], out=want[:S], layout="SHD", scale=128 ** -0.5,
                blocks=bl.on(dev), q_norm=wq, k_norm=wk, eps=EPS, rope_table=tab)
    torch.cuda.synchronize()
    lo, hi = rank * n, min(S, (rank + 1) * n)
    q_out.put((rank, (out[: hi - lo].float() - want[lo:hi].float()).abs().max().item()))


@pytest.mark.parametrize("chunks", [1, 3])
def test_c_abi_seqshard_two_gpus(gpu, chunks):
    """h3c_comm_init + h3c_attn_fwd_seqshard (NCCL grouped send/recv inside
    the library) on 2 GPUs equals the single-GPU fused call, unpipelined and
    pipelined over 3 uneven head chunks (4 heads per rank)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q, id_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_abi_worker, args=(r, 2, id_q, q, chunks)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=120) for _ in range(2)]
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, err in res:
        assert err == 0.0, (rank, err)


def _timeout_worker(rank, world, id_q, q_out, done_q):
    try:
        _timeout_body(rank, world, id_q, q_out, done_q)
    except Exception as e:  # report instead of leaving the parent waiting
        q_out.put((rank, repr(e)))


def _timeout_body(rank, world, id_q, q_out, done_q):
    import sys
    import time

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "minimax-h3-swift_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    from h3attention import BlockList, H3CError, Runtime, _lib
    from h3attention.configs import CONFIGS
    from h3attention.sharding import seq_shard_len

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    wl = CONFIGS["config1"]
    S, H = wl.seq_len, wl.heads
    rt = Runtime.get(rank)
    if rank == 0:  # rank 0 creates the NCCL id and hands it to rank 1
        uid = Runtime.comm_unique_id()
        id_q.put(uid)
    else:
        uid = id_q.get(timeout=60)
    n = seq_shard_len(S, world)
    mine = [rt.fill_normal(torch.empty((n, H, 128), dtype=torch.bfloat16, device=dev), 7 + rank, st)
            for st in (1, 2, 3)]
    bl = BlockList.build(wl.mask_spec())
    rt.comm_init(uid, world, rank)
    out = torch.empty_like(mine[0])
    kw = dict(q=mine[0], k=mine[1], v=mine[2], out=out, layout="SHD", scale=128 ** -0.5, blocks=bl.on(dev),
              seq_len=S)
    # step 1: both ranks take part; the bounded wait returns in time
    rt.attn_fwd_seqshard(timeout_ms=60000, **kw)
    if rank == 1:
        # this rank leaves between steps: it never joins step 2 and waits
        # (alive, its memory intact) until rank 0 has reported
        q_out.put((1, "left after step 1"))
        done_q.get(timeout=120)
        os._exit(0)
    # step 2 on rank 0 alone: the exchange cannot complete; the wait must
    # give up after 2 s with H3C_ERR_TIMEOUT (communicator aborted)
    t0 = time.time()
    status = None
    try:
        rt.attn_fwd_seqshard(timeout_ms=2000, **kw)
    except H3CError as e:
        status = e.status
    waited = time.time() - t0
    # the context stays usable for the single-GPU call
    want = torch.empty_like(mine[0])
    rt.attn_fwd(q=mine[0], k=mine[1], v=mine[2], out=want, layout="SHD", scale=128 ** -0.5, blocks=bl.on(dev))
    torch.cuda.synchronize()
    rt.device_status()
    ok_after = bool(torch.isfinite(want.float()).all().item())
    rt.comm_destroy()
    q_out.put((0, (status, waited, ok_after, _lib.H3C_ERR_TIMEOUT)))


def test_c_abi_seqshard_peer_that_never_joins_times_out(gpu):
    """Failure detection of the NCCL exchange without a GPU fault: rank 1
    takes part in one step and then never joins the next (it stays alive).
    Rank 0's bounded wait (h3c_comm_wait) gives up after 2 s, aborts the
    communicator and reports H3C_ERR_TIMEOUT; the context still runs the
    single-GPU call.  NVLS off, plain NCCL send/recv."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q, id_q, done_q = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, id_q, q, done_q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=180) for _ in range(2))
    finally:
        done_q.put("done")
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[1] == "left after step 1", res
    status, waited, ok_after, timeout_code = res[0]
    assert status == timeout_code, res
    assert 1.5 <= waited <= 30.0, waited
    assert ok_after
