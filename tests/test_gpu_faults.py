"""Failure detection without a GPU fault: the host drops one K/V load (a
test hook read from the environment), so the kernel's bounded mbarrier waits
run out after a short limit; the call must come back as H3C_ERR_TIMEOUT, and
the same context must then produce correct results again."""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a, dev):
    import torch

    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)


def test_dropped_load_times_out_and_context_recovers(gpu):
    import torch

    from h3attention import BlockList, H3CError, MaskSpec, Runtime, _lib

    S, H = 1024, 2
    rt = Runtime.get(0)
    spec = MaskSpec(seq_len=S, frames=4, height=16, width=16, n_random=1, seed=3)
    bl = BlockList.build(spec)
    q, k, v = (O.fill_normal_bf16((S, H, 128), 12, st) for st in (1, 2, 3))
    qd, kd, vd = (_dev(a, gpu) for a in (q, k, v))
    out = torch.empty_like(qd)
    kw = dict(q=qd, k=kd, v=vd, out=out, layout="SHD", scale=128 ** -0.5, blocks=bl.on(gpu))
    os.environ["H3C_TEST_DROP_ITEM"] = "3"
    os.environ["H3C_TEST_WAIT_LIMIT_NS"] = "50000000"  # 50 ms
    try:
        with pytest.raises(H3CError) as ei:
            rt.attn_fwd_sync(**kw)
        assert ei.value.status == _lib.H3C_ERR_TIMEOUT
    finally:
        del os.environ["H3C_TEST_DROP_ITEM"]
        del os.environ["H3C_TEST_WAIT_LIMIT_NS"]
    rt.device_status()  # cleared by the failing call
    rt.attn_fwd_sync(**kw)
    want = O.attend_streaming(q, k, v, bl.row_ptr, bl.col_idx)
    got = out.float().cpu().numpy().transpose(1, 0, 2)
    err = np.abs(got - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3
