"""CUDA path vs the CPU checker, through the C ABI (B200 only).

Tolerances: integer and generator work is bit-exact; the prologue is within
one bf16 ulp (reduction order of the fp32 sum of squares; the reference's own
bound is relRMS < 1e-3 and worst < 8 ulp, QKFusionTests.swift:109-110);
attention on unit-variance inputs is max-abs <= 2e-2 and mean-abs <= 2e-3
against the fp32 restatement.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _t(a, dev):
    import torch

    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)


def _np(t):
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _rt():
    from h3attention import Runtime

    return Runtime.get(0)


def _spec(**kw):
    from h3attention import MaskSpec

    return MaskSpec(**kw)


def _check_attn(got_bf16_shd, want_hsd, rows=None):
    got = O.bf16_to_f32(got_bf16_shd).transpose(1, 0, 2)
    if rows is not None:
        got, want_hsd = got[:, rows], want_hsd[:, rows]
    err = np.abs(got - want_hsd)
    assert np.isfinite(got).all()
    assert err.max() <= MAX_ABS, f"max-abs {err.max()}"
    assert err.mean() <= MEAN_ABS, f"mean-abs {err.mean()}"
    return float(err.max()), float(err.mean())


# --------------------------------------------------------------- aux kernels
def test_fill_normal_matches_checker(gpu):
    import torch

    out = torch.empty(1 << 20, dtype=torch.bfloat16, device=gpu)
    _rt().fill_normal(out, 1234, 3)
    torch.cuda.synchronize()
    ref = O.fill_normal_bf16((1 << 20,), 1234, 3)
    assert np.count_nonzero(_np(out) != ref) <= 2


def test_rope_table_matches_checker(gpu):
    import torch

    from h3attention.configs import CONFIGS

    pos = CONFIGS["config1"].positions()
    tab = _rt().rope_table(torch.from_numpy(pos).to(gpu))
    ref = O.rope_table(pos)
    diff = np.abs(_np(tab).astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and np.count_nonzero(diff) <= 4


@pytest.mark.parametrize("S,H,half", [(4096, 8, 64), (1000, 3, 48), (777, 2, 46), (257, 2, 0)])
def test_prologue_matches_checker(gpu, S, H, half):
    import torch

    x = O.fill_normal_bf16((S, H, 128), 21, 1)
    w = O.fill_normal_bf16((128,), 21, 4, 1.0, 0.02)
    if half:
        dims = {64: (32, 48, 48), 48: (32, 32, 32), 46: (30, 32, 30)}[half]
        pos = np.stack([np.arange(S) % 17, np.arange(S) % 13, np.arange(S) % 11], 1).astype(np.int32)
        tab = O.rope_table(pos, dims=dims)
    else:
        tab = None
    ref = O.prologue(x, w, 1e-6, tab)
    xd = _t(x, gpu)
    out = torch.empty_like(xd)
    _rt().prologue(xd, out, _t(w, gpu), 1e-6, None if tab is None else _t(tab, gpu))
    torch.cuda.synchronize()
    got = _np(out)
    g, r = O.bf16_to_f32(got), O.bf16_to_f32(ref)
    if tab is None:  # RMSNorm alone: one rounding of a correctly ordered product
        assert np.abs(got.astype(np.int32) - ref.astype(np.int32)).max() <= 1
    # the reference's gate (QKFusionTests.swift:67-110): relRMS < 1e-3 and a
    # worst error, scaled by |ref| + rms, under 8 bf16 ulp (2^-7 each)
    rms = np.sqrt(np.mean(r ** 2))
    assert np.sqrt(np.mean((g - r) ** 2)) / rms < 1e-3
    assert np.max(np.abs(g - r) / (np.abs(r) + rms)) / 0.0078125 < 8


MASKS = [
    dict(seq_len=4096, frames=16, height=16, width=16, n_random=2, seed=1),
    dict(seq_len=125632, prefix_len=640, frames=31, height=48, width=84, radius_h=2, radius_w=2, n_random=4, seed=3),
    dict(seq_len=800, prefix_len=100, frames=7, height=10, width=10, n_random=50, seed=5),
]


@pytest.mark.parametrize("kw", MASKS)
def test_device_blockmask_bit_identical(gpu, kw):
    rp, ci = _rt().blockmask_device(_spec(**kw), capacity=400000)
    wrp, wci = O.blockmask_build(O.mask_spec(**kw))
    assert np.array_equal(rp.cpu().numpy(), wrp) and np.array_equal(ci.cpu().numpy(), wci)


# ----------------------------------------------------------------- attention
def _case(S, H, spec_kw, seed=4):
    q, k, v = (O.fill_normal_bf16((S, H, 128), seed, st) for st in (1, 2, 3))
    rp, ci = O.blockmask_build(O.mask_spec(**spec_kw))
    return q, k, v, rp, ci


ATTN_CASES = {
    "config1": (4096, 8, dict(seq_len=4096, frames=16, height=16, width=16, n_random=2, seed=1)),
    "ragged_odd_heads": (1000, 3, dict(seq_len=1000, frames=10, height=10, width=10, n_random=1, seed=2)),
    "prefix": (1640, 2, dict(seq_len=1640, prefix_len=640, frames=10, height=10, width=10, n_random=1, seed=3)),
    "one_block": (77, 1, dict(seq_len=77, frames=7, height=1, width=11)),
    "dense_ragged": (1500, 2, dict(seq_len=1500, prefix_len=1500, frames=0, height=0, width=0)),
}


@pytest.mark.parametrize("kernel", ["mma_sync", "tcgen05"])
@pytest.mark.parametrize("name", list(ATTN_CASES))
def test_attention_matches_checker(gpu, kernel, name):
    import torch

    from h3attention import _lib

    S, H, kw = ATTN_CASES[name]
    q, k, v, rp, ci = _case(S, H, kw)
    want = O.attend_streaming(q, k, v, rp, ci)
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    blocks = (torch.from_numpy(rp).to(gpu), torch.from_numpy(ci).to(gpu))
    flags = _lib.H3C_KERNEL_MMA_SYNC if kernel == "mma_sync" else 0
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=out, layout="SHD", scale=1 / np.sqrt(128), blocks=blocks, flags=flags)
    torch.cuda.synchronize()
    _check_attn(_np(out), want)


@pytest.mark.parametrize("kernel", ["mma_sync", "tcgen05"])
def test_growing_scores_exercise_the_rescale(gpu, kernel):
    """Keys whose magnitude grows block by block make the row max jump by
    more than 2^8 several times along a row, so the lazy rescale of O and l
    (and, in the tcgen05 kernel, the recomputation of a block's
    exponentials after the max moved) runs on every row."""
    import torch

    from h3attention import _lib

    S, H = 2048, 2
    q, k, v, rp, ci = _case(S, H, dict(seq_len=S, prefix_len=S, frames=0, height=0, width=0))
    kf = O.bf16_to_f32(k).reshape(S // 128, 128, H, 128) * (1.0 + 1.5 * np.arange(S // 128))[:, None, None, None]
    k = O.f32_to_bf16(kf.reshape(S, H, 128).astype(np.float32))
    want = O.attend_streaming(q, k, v, rp, ci)
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    blocks = (torch.from_numpy(rp).to(gpu), torch.from_numpy(ci).to(gpu))
    flags = _lib.H3C_KERNEL_MMA_SYNC if kernel == "mma_sync" else 0
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=out, layout="SHD", scale=1 / np.sqrt(128), blocks=blocks, flags=flags)
    torch.cuda.synchronize()
    _check_attn(_np(out), want)


@pytest.mark.parametrize("kernel", ["mma_sync", "tcgen05"])
def test_empty_rows_give_zeros(gpu, kernel):
    """A caller-supplied block list may leave query blocks without any kept
    key block; their rows come out as zeros (O / max(l, 1e-30) with l = 0),
    as in the checker.  Row 1 empties one tile of a two-tile CTA, rows 4-5
    a whole CTA, and the last row a single-tile CTA."""
    import torch

    from h3attention import _lib

    S, H = 1100, 2
    q, k, v, rp, ci = _case(S, H, dict(seq_len=S, frames=11, height=10, width=10, n_random=1, seed=6))
    rows = [ci[rp[i]:rp[i + 1]] for i in range(len(rp) - 1)]
    for i in (1, 4, 5, len(rows) - 1):
        rows[i] = rows[i][:0]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.concatenate(rows).astype(np.int32)
    want = O.attend_streaming(q, k, v, rp, ci)
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    blocks = (torch.from_numpy(rp).to(gpu), torch.from_numpy(ci).to(gpu))
    flags = _lib.H3C_KERNEL_MMA_SYNC if kernel == "mma_sync" else 0
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=out, layout="SHD", scale=1 / np.sqrt(128), blocks=blocks, flags=flags)
    torch.cuda.synchronize()
    got = _np(out)
    for i in (1, 4, 5, len(rows) - 1):
        assert np.all(got[i * 128:min(S, i * 128 + 128)] == 0), i
    _check_attn(got, want)


@pytest.mark.parametrize("kernel", ["mma_sync", "tcgen05"])
def test_fused_prologue_matches_checker(gpu, kernel):
    import torch

    from h3attention import _lib
    from h3attention.configs import CONFIGS

    wl = CONFIGS["config1"]
    S, H = wl.seq_len, wl.heads
    q, k, v = (O.fill_normal_bf16((S, H, 128), 9, st) for st in (1, 2, 3))
    wq, wk = (O.fill_normal_bf16((128,), 9, st, 1.0, 0.02) for st in (4, 5))
    tab = O.rope_table(wl.positions())
    rp, ci = O.blockmask_build(O.mask_spec(seq_len=S, frames=16, height=16, width=16, n_random=2, seed=wl.seed))
    want = O.attend_streaming(O.prologue(q, wq, 1e-6, tab), O.prologue(k, wk, 1e-6, tab), v, rp, ci)
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    out = torch.empty_like(qd)
    blocks = (torch.from_numpy(rp).to(gpu), torch.from_numpy(ci).to(gpu))
    flags = _lib.H3C_KERNEL_MMA_SYNC if kernel == "mma_sync" else 0
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=out, layout="SHD", scale=1 / np.sqrt(128), blocks=blocks, flags=flags,
                   q_norm=_t(wq, gpu), k_norm=_t(wk, gpu), eps=1e-6, rope_table=_t(tab, gpu))
    torch.cuda.synchronize()
    _check_attn(_np(out), want)


def test_fused_norm_without_rope(gpu):
    """The fused call without a RoPE table (AttentionLayer runs RoPE only when
    the render has a table, DiTBlock.swift:349-352): RMSNorm alone on q and k
    (H3C_NO_ROPE), against the checker."""
    import torch

    S, H = 1500, 3
    q, k, v, rp, ci = _case(S, H, dict(seq_len=S, frames=15, height=10, width=10, n_random=1, seed=9))
    wq, wk = (O.fill_normal_bf16((128,), 9, st, 1.0, 0.02) for st in (4, 5))
    want = O.attend_streaming(O.prologue(q, wq, 1e-6, None), O.prologue(k, wk, 1e-6, None), v, rp, ci)
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    out = torch.empty_like(qd)
    blocks = (torch.from_numpy(rp).to(gpu), torch.from_numpy(ci).to(gpu))
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=out, layout="SHD", scale=1 / np.sqrt(128), blocks=blocks,
                   q_norm=_t(wq, gpu), k_norm=_t(wk, gpu), eps=1e-6, rope_table=None)
    torch.cuda.synchronize()
    _check_attn(_np(out), want)


def test_hsd_layout_and_head_shard(gpu):
    """The seam's [H,S,D] layout, and a head shard [1, 3) of 4 heads."""
    import torch

    S, H = 600, 4
    q, k, v, rp, ci = _case(S, H, dict(seq_len=600, frames=6, height=10, width=10, n_random=1, seed=8))
    want = O.attend_streaming(q, k, v, rp, ci)
    qd, kd, vd = (_t(np.ascontiguousarray(a.transpose(1, 0, 2)), gpu) for a in (q, k, v))
    out = torch.zeros_like(qd)
    blocks = (torch.from_numpy(rp).to(gpu), torch.from_numpy(ci).to(gpu))
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=out, layout="HSD", scale=1 / np.sqrt(128), blocks=blocks, head_offset=1,
                   head_count=2)
    torch.cuda.synchronize()
    got = _np(out.transpose(0, 1))
    _check_attn(got[:, 1:3], want[1:3])
    assert np.all(_np(out)[[0, 3]] == 0), "heads outside the shard are untouched"


@pytest.mark.parametrize("name,qbs", [("config2", [0, 1, 488, 975, 976]), ("config3", [0, 4, 5, 6, 500, 981])])
def test_full_size_config2_sampled(gpu, name, qbs):
    """Configs 2 and 3 at full size (S=124,992 / 125,632, H=40) on the
    tcgen05 kernel, checked on a deterministic sample of query blocks (for
    config 3: dense audio rows 0-4 and the first video rows) and heads."""
    import torch

    from h3attention import BlockList, Runtime
    from h3attention.configs import CONFIGS

    wl = CONFIGS[name]
    S, H = wl.seq_len, wl.heads
    rt = Runtime.get(0)
    q, k, v = (rt.fill_normal(torch.empty((S, H, 128), dtype=torch.bfloat16, device=gpu), wl.seed, st)
               for st in (1, 2, 3))
    bl = BlockList.build(wl.mask_spec())
    out = torch.empty_like(q)
    rt.attn_fwd(q=q, k=k, v=v, out=out, layout="SHD", scale=1 / np.sqrt(128), blocks=bl.on(gpu))
    torch.cuda.synchronize()
    heads = (17, 19)
    qh, kh, vh = (_np(t[:, heads[0]:heads[1]]) for t in (q, k, v))
    want = O.attend_streaming(qh, kh, vh, bl.row_ptr, bl.col_idx, qblocks=qbs)
    rows = np.concatenate([np.arange(b * 128, min(S, b * 128 + 128)) for b in qbs])
    _check_attn(_np(out[:, heads[0]:heads[1]]), want, rows=rows)


def test_host_pipeline_matches_device_call(gpu):
    """h3attention.host.HostAttention (pinned host [H,S,D] in/out, head
    chunks overlapped on three streams) equals the device call."""
    import torch

    from h3attention import BlockList, MaskSpec, Runtime
    from h3attention.host import HostAttention

    S, H = 2000, 6
    spec = MaskSpec(seq_len=S, frames=5, height=20, width=20, n_random=2, seed=4)
    bl = BlockList.build(spec)
    q, k, v = (O.fill_normal_bf16((H, S, 128), 17, st) for st in (1, 2, 3))
    wq, wk = (_t(O.fill_normal_bf16((128,), 17, st, 1.0, 0.02), gpu) for st in (4, 5))
    pos = np.stack([np.arange(S) // 400, (np.arange(S) // 20) % 20, np.arange(S) % 20], 1).astype(np.int32)
    tab = _t(O.rope_table(pos), gpu)
    hq, hk, hv = (torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).pin_memory() for a in (q, k, v))
    hout = torch.empty_like(hq).pin_memory()
    ha = HostAttention(0, H, S, chunk_heads=4)
    ha(hq, hk, hv, hout, bl.on(gpu), 128 ** -0.5, q_norm=wq, k_norm=wk, eps=1e-6, rope_table=tab)
    torch.cuda.synchronize()
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    want = torch.empty_like(qd)
    _rt().attn_fwd(q=qd, k=kd, v=vd, out=want, layout="HSD", scale=128 ** -0.5, blocks=bl.on(gpu), q_norm=wq,
                   k_norm=wk, eps=1e-6, rope_table=tab)
    torch.cuda.synchronize()
    assert torch.equal(hout, want.cpu())


def test_backend_seam_fused_and_decline(gpu):
    """The seam mirror: CUDABackend.attend_fused equals prologue + attend;
    a call outside the prepared layout is declined (None) and sdpa() then
    runs the dense path, which equals the backend with every block kept."""
    import torch

    from h3attention import AttentionContext, AttentionRegistry, Machine, MaskSpec, sdpa

    S, H = 1024, 2
    sel = AttentionRegistry.resolve("b200-block-sparse", Machine.detect())
    spec = MaskSpec(seq_len=S, frames=4, height=16, width=16, n_random=1, seed=9)
    sel.backend.prepare_render(spec)
    ctx = AttentionContext(block_index=3, block_count=50, schedule_progress=0.5, sequence_length=S,
                           video_span=(0, S))
    q, k, v = (O.fill_normal_bf16((H, S, 128), 23, st) for st in (1, 2, 3))
    wq, wk = (O.fill_normal_bf16((128,), 23, st, 1.0, 0.02) for st in (4, 5))
    pos = np.stack([np.arange(S) // 256, (np.arange(S) // 16) % 16, np.arange(S) % 16], 1).astype(np.int32)
    tab = O.rope_table(pos)
    qd, kd, vd = (_t(a, gpu) for a in (q, k, v))
    fused = sel.backend.attend_fused(qd, kd, vd, 128 ** -0.5, _t(wq, gpu), _t(wk, gpu), 1e-6, _t(tab, gpu), ctx)
    qs, ks = (O.prologue(np.ascontiguousarray(a.transpose(1, 0, 2)), w, 1e-6, tab) for a, w in ((q, wq), (k, wk)))
    unfused = sel.backend.attend(_t(np.ascontiguousarray(qs.transpose(1, 0, 2)), gpu),
                                 _t(np.ascontiguousarray(ks.transpose(1, 0, 2)), gpu), vd, 128 ** -0.5, None, ctx)
    torch.cuda.synchronize()
    d = (fused.float() - unfused.float()).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3
    # decline: a sequence the render was not prepared for
    other = AttentionContext(3, 50, 0.5, S // 2, None)
    half = [t[:, : S // 2] for t in (qd, kd, vd)]
    assert sel.backend.attend(*half, 128 ** -0.5, None, other) is None
    # sdpa() with a declining call runs the dense path ([S,H,D] in, [S,H*D] out)
    shd = [t.transpose(0, 1) for t in half]
    dense = sdpa(*shd, head_dim=128, backend=sel.backend, context=other)
    assert dense.shape == (S // 2, H * 128)
    want = O.attend_dense_f64(*(np.ascontiguousarray(a[:, : S // 2].transpose(1, 0, 2)) for a in (q, k, v)))
    got = dense.float().cpu().numpy().reshape(S // 2, H, 128).transpose(1, 0, 2)
    assert np.abs(got - want).max() <= 2e-2


@pytest.mark.parametrize("vendor", ["blocked", "interleaved"])
def test_qkv_direct_views(gpu, vendor):
    """q, k, v read straight from one [S, 3*H*D] QKV GEMM output through
    strided views, with the fused prologue: equals the call on split copies.
    Both checkpoint layouts of attn.qkv_proj (FRAGILE_CONTRACTS.md section 9)
    are views: Comfy-Org's blocked (3, heads, headDim) Q|K|V
    (DiTBlock.swift:338-344) and DeepBeepMeep's per-head interleaved
    (heads, 3, headDim), so neither needs the permute-on-load."""
    import torch

    from h3attention import BlockList, MaskSpec
    from h3attention._lib import View

    S, H = 1500, 3
    qkv = _t(O.fill_normal_bf16((S, 3 * H * 128), 31, 1), gpu)
    wq, wk = (_t(O.fill_normal_bf16((128,), 31, st, 1.0, 0.02), gpu) for st in (4, 5))
    pos = np.stack([np.arange(S) // 300, (np.arange(S) // 20) % 15, np.arange(S) % 20], 1).astype(np.int32)
    tab = _t(O.rope_table(pos), gpu)
    bl = BlockList.build(MaskSpec(seq_len=S, frames=5, height=15, width=20, n_random=1, seed=2))
    if vendor == "blocked":
        views = [qkv[:, i * H * 128:(i + 1) * H * 128].view(S, H, 128) for i in range(3)]  # strided, no copy
        assert views[0].stride() == (3 * H * 128, 128, 1)
    else:
        per_head = qkv.view(S, H, 3, 128)
        views = [per_head[:, :, i] for i in range(3)]
        assert views[0].stride() == (3 * H * 128, 3 * 128, 1)
    out_v = torch.empty((S, H, 128), dtype=torch.bfloat16, device=gpu)
    _rt().attn_fwd(q=views[0], k=views[1], v=views[2], out=out_v, layout="SHD", scale=128 ** -0.5,
                   blocks=bl.on(gpu), q_norm=wq, k_norm=wk, eps=1e-6, rope_table=tab)
    copies = [t.contiguous() for t in views]
    out_c = torch.empty_like(out_v)
    _rt().attn_fwd(q=copies[0], k=copies[1], v=copies[2], out=out_c, layout="SHD", scale=128 ** -0.5,
                   blocks=bl.on(gpu), q_norm=wq, k_norm=wk, eps=1e-6, rope_table=tab)
    torch.cuda.synchronize()
    assert torch.equal(out_v, out_c)
