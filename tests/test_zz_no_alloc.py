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
