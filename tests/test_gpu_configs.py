"""The exact call bench.py times, at every benchmark configuration, against
the CPU checker (B200 only).

Each case builds the inputs the way bench.py does (the seeded device
generator at full size, H = 40), makes the fused call through the C ABI
(h3c_attn_fwd with H3C_FUSE_PROLOGUE: RMSNorm + RoPE + block-sparse
attention), and checks a deterministic sample of query blocks of two heads
against the oracle, which normalises and rotates those heads over the whole
sequence with its own RoPE table and runs the streaming attention of
Sources/H3Attention/AxialReference.swift:129-171.  The error is taken per
query block, never averaged across blocks (the reference's rule,
Tests/H3AttentionTests/AxialMeasureTests.swift:20-27).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3

CASES = ["config1", "config2", "config3", "config4", "config5@0.05", "config5@0.1", "config5@0.25", "config5@0.5",
         "production"]


def _np(t):
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_table(wl):
    if wl.render:
        from h3attention.configs import shared_inv_freq

        text, width, height, length = wl.render
        _, pos = O.packed_layout(text, O.latent_geometry(width, height, length))
        return O.rope_table_shared(pos.astype(np.float32), shared_inv_freq())
    return O.rope_table(wl.positions())


@pytest.mark.parametrize("name", CASES)
def test_bench_call_matches_checker(gpu, name):
    import torch

    import bench
    from h3attention import BlockList, Runtime, torchref
    from h3attention.configs import STREAM_K, STREAM_Q, STREAM_V, STREAM_WK, STREAM_WQ

    wl = bench._workload(name)
    S, H = wl.seq_len, wl.heads
    rt = Runtime.get(0)
    bf = torch.bfloat16

    def fill(shape, stream, mean=0.0, std=1.0):
        return rt.fill_normal(torch.empty(shape, dtype=bf, device=gpu), wl.seed, stream, mean, std)

    q, k, v = (fill((S, H, 128), st) for st in (STREAM_Q, STREAM_K, STREAM_V))
    wq, wk = fill((128,), STREAM_WQ, 1.0, 0.02), fill((128,), STREAM_WK, 1.0, 0.02)
    tab = wl.rope_table(rt, gpu)
    bl = BlockList.build(wl.mask_spec())
    out = torch.full_like(q, float("nan"))
    args = rt.attn_args(q, k, v, out, "SHD", 128 ** -0.5, bl.on(gpu), q_norm=wq, k_norm=wk, eps=wl.eps,
                        rope_table=tab)
    rt.attn_fwd_args(args)
    torch.cuda.synchronize()
    rt.device_status()

    heads = [3, H - 1]
    qbs = torchref.sample_blocks(bl.n_blocks, 5, seed=len(name))
    if wl.audio:  # the dense prefix rows and the first video rows
        qbs = sorted(set(qbs) | {0, wl.audio // 128, wl.audio // 128 + 1})
    table = _oracle_table(wl)
    wq_h, wk_h = _np(wq), _np(wk)
    worst = (0.0, 0.0)
    for h in heads:
        qh, kh, vh = (_np(t[:, h:h + 1]) for t in (q, k, v))
        qn, kn = O.prologue(qh, wq_h, wl.eps, table), O.prologue(kh, wk_h, wl.eps, table)
        want = O.attend_streaming(qn, kn, vh, bl.row_ptr, bl.col_idx, qblocks=qbs)[0]
        got = O.bf16_to_f32(_np(out[:, h]))
        for b in qbs:
            r0, r1 = b * 128, min(S, b * 128 + 128)
            err = np.abs(got[r0:r1] - want[r0:r1])
            assert np.isfinite(got[r0:r1]).all(), (name, h, b)
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (name, h, b, err.max(), err.mean())
            worst = (max(worst[0], err.max()), max(worst[1], err.mean()))
    print(f"{name}: S={S} H={H} density {bl.density:.4f}; worst per-block max-abs {worst[0]:.3e} "
          f"mean-abs {worst[1]:.3e}")
    del q, k, v, out
    torch.cuda.empty_cache()
