"""The allocation-free entry point h3c_attn_fwd_noalloc, through the C ABI.

Some callers may not call cudaMalloc: a host whose framework has taken the
device heap into its own pool, or a loop where an allocation at call time is
not acceptable.  For them the library offers the fused prologue + attention
with its scratch in a fixed device array inside the library.  This test
checks, on two calls in a row, that its output agrees with the ordinary
h3c_attn_fwd (same tolerance as the other attention tests), and that a call
needing more than the fixed scratch is refused.  The file is named so that
pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _dev(a, dev):
    import torch

    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)


def test_noalloc_matches_attn_fwd_twice(gpu):
    import torch

    from h3attention import BlockList, MaskSpec, Runtime, _lib
    from h3attention.configs import CONFIGS

    L = _lib.load()
    wl = CONFIGS["config1"]
    S, H = wl.seq_len, wl.heads
    rt = Runtime.get(0)
    torch.cuda.set_device(0)
    bl = BlockList.build(MaskSpec(seq_len=S, frames=16, height=16, width=16, n_random=2, seed=wl.seed))
    blocks = bl.on(gpu)
    tab = _dev(O.rope_table(wl.positions()), gpu)
    err = C.create_string_buffer(512)
    for call in range(2):
        q, k, v = (_dev(O.fill_normal_bf16((S, H, 128), 30 + call, st), gpu) for st in (1, 2, 3))
        wq, wk = (_dev(O.fill_normal_bf16((128,), 30 + call, st, 1.0, 0.02), gpu) for st in (4, 5))
        want = torch.empty_like(q)
        rt.attn_fwd(q=q, k=k, v=v, out=want, layout="SHD", scale=128 ** -0.5, blocks=blocks,
                    q_norm=wq, k_norm=wk, eps=1e-6, rope_table=tab)
        got = torch.full_like(q, float("nan"))
        args = rt.attn_args(q, k, v, got, "SHD", 128 ** -0.5, blocks, q_norm=wq, k_norm=wk, eps=1e-6,
                            rope_table=tab)
        st = L.h3c_attn_fwd_noalloc(C.byref(args), torch.cuda.current_stream().cuda_stream or None, err, len(err))
        assert st == _lib.H3C_OK, err.value.decode()
        torch.cuda.synchronize()
        d = (got.float() - want.float()).abs()
        assert torch.isfinite(got.float()).all()
        assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, (call, d.max().item(), d.mean().item())


def test_noalloc_refuses_beyond_its_scratch(gpu):
    import torch

    from h3attention import BlockList, Runtime, _lib

    L = _lib.load()
    rt = Runtime.get(0)
    S, H = 8192, 9  # 8192 x 9 token-heads > 65536
    x = torch.zeros((S, H, 128), dtype=torch.bfloat16, device=gpu)
    w = torch.ones(128, dtype=torch.bfloat16, device=gpu)
    bl = BlockList.dense(S)
    args = rt.attn_args(x, x, x, torch.empty_like(x), "SHD", 0.1, bl.on(gpu), q_norm=w, k_norm=w, eps=1e-6)
    err = C.create_string_buffer(512)
    st = L.h3c_attn_fwd_noalloc(C.byref(args), None, err, len(err))
    assert st == _lib.H3C_ERR_CAPACITY
    assert b"limit" in err.value


def _noalloc(L, args, err):
    import torch

    return L.h3c_attn_fwd_noalloc(C.byref(args), torch.cuda.current_stream().cuda_stream or None, err, len(err))


@pytest.mark.parametrize("case", ["head_range", "no_rope"])
def test_noalloc_head_range_and_rmsnorm_only(gpu, case):
    """A head sub-range (offsets into q/k/v/out, scratch sized by head_count)
    and the RMSNorm-only prologue, both equal to h3c_attn_fwd; the error
    buffer stays empty and the status word clean on success."""
    import torch

    from h3attention import BlockList, MaskSpec, Runtime, _lib
    from h3attention.configs import CONFIGS

    L = _lib.load()
    wl = CONFIGS["config1"]
    S, H = wl.seq_len, wl.heads
    rt = Runtime.get(0)
    bl = BlockList.build(MaskSpec(seq_len=S, frames=16, height=16, width=16, n_random=2, seed=wl.seed))
    blocks = bl.on(gpu)
    tab = None if case == "no_rope" else _dev(O.rope_table(wl.positions()), gpu)
    ho, hc = (3, 4) if case == "head_range" else (0, H)
    q, k, v = (_dev(O.fill_normal_bf16((S, H, 128), 40, st), gpu) for st in (1, 2, 3))
    wq, wk = (_dev(O.fill_normal_bf16((128,), 40, st, 1.0, 0.02), gpu) for st in (4, 5))
    want = torch.zeros_like(q)
    rt.attn_fwd(q=q, k=k, v=v, out=want, layout="SHD", scale=128 ** -0.5, blocks=blocks, head_offset=ho,
                head_count=hc, q_norm=wq, k_norm=wk, eps=1e-6, rope_table=tab)
    got = torch.zeros_like(q)
    args = rt.attn_args(q, k, v, got, "SHD", 128 ** -0.5, blocks, head_offset=ho, head_count=hc, q_norm=wq,
                        k_norm=wk, eps=1e-6, rope_table=tab)
    err = C.create_string_buffer(512)
    assert _noalloc(L, args, err) == _lib.H3C_OK, err.value.decode()
    assert err.value == b""
    torch.cuda.synchronize()
    assert L.h3c_attn_fwd_noalloc_status() == _lib.H3C_OK
    d = (got.float() - want.float()).abs()
    assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS
    outside = [h for h in range(H) if not ho <= h < ho + hc]
    assert all(torch.count_nonzero(got[:, h]).item() == 0 for h in outside), "heads outside the range untouched"


def test_noalloc_reports_a_timeout(gpu):
    """A dropped K/V load (host-side test hook) makes the bounded waits run
    out: the call itself returns H3C_OK (it is asynchronous), the status
    word then reports H3C_ERR_TIMEOUT once, and the next call is correct."""
    import os

    import torch

    from h3attention import BlockList, MaskSpec, Runtime, _lib

    L = _lib.load()
    rt = Runtime.get(0)
    S, H = 1024, 2
    bl = BlockList.build(MaskSpec(seq_len=S, frames=4, height=16, width=16, n_random=1, seed=3))
    q, k, v = (_dev(O.fill_normal_bf16((S, H, 128), 12, st), gpu) for st in (1, 2, 3))
    w = torch.ones(128, dtype=torch.bfloat16, device=gpu)
    out = torch.empty_like(q)
    args = rt.attn_args(q, k, v, out, "SHD", 128 ** -0.5, bl.on(gpu), q_norm=w, k_norm=w, eps=1e-6)
    err = C.create_string_buffer(512)
    os.environ["H3C_TEST_DROP_ITEM"] = "3"
    os.environ["H3C_TEST_WAIT_LIMIT_NS"] = "50000000"  # 50 ms
    try:
        assert _noalloc(L, args, err) == _lib.H3C_OK, err.value.decode()
    finally:
        del os.environ["H3C_TEST_DROP_ITEM"]
        del os.environ["H3C_TEST_WAIT_LIMIT_NS"]
    assert L.h3c_attn_fwd_noalloc_status() == _lib.H3C_ERR_TIMEOUT
    assert L.h3c_attn_fwd_noalloc_status() == _lib.H3C_OK  # read and cleared
    assert _noalloc(L, args, err) == _lib.H3C_OK
    assert L.h3c_attn_fwd_noalloc_status() == _lib.H3C_OK
    want = torch.empty_like(q)
    rt.attn_fwd(q=q, k=k, v=v, out=want, layout="SHD", scale=128 ** -0.5, blocks=bl.on(gpu), q_norm=w, k_norm=w,
                eps=1e-6)
    torch.cuda.synchronize()
    d = (out.float() - want.float()).abs()
    assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS
