"""The CPU checker pinned against the reference's own known answers and
identities (Tests/H3AttentionTests/AxialReferenceTests.swift,
Tests/H3ModulesTests/QKFusionTests.swift).  No GPU."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "axial_reference.json")))


def _topology(g):
    s = g["prefix"] + g["frames"] * g["height"] * g["width"]
    return O.AxialTopology(s, (g["prefix"], s), g["frames"], g["height"], g["width"], g["landmarks"])


# ------------------------------------------------------- AxialTopology pins
def test_topology_spot_checks():
    t = _topology(GOLD["fixture"])
    sp = GOLD["spot"]
    assert list(t.locate(sp["query"])) == sp["locate"]
    for k in sp["allowed"]:
        assert t.allows(sp["query"], k)
    for k in sp["excluded"]:
        assert not t.allows(sp["query"], k)
    assert all(t.allows(0, k) for k in range(t.video_span[1]))


def test_density_counted_equals_closed_form():
    t = _topology(GOLD["density_fixture"])
    m = t.mask_rows(range(t.video_span[1]))
    counted = float((m == 0).sum()) / m.size
    assert abs(counted - t.density) < 1e-9


def test_geometry_refusal_and_landmarks():
    g = GOLD["geometry"]
    lt, lh, lw = g["latent_t"], g["latent_h"], g["latent_w"]
    assert O.AxialTopology.from_geometry(g["seq_len"], tuple(g["video_ok"]), lt, lh, lw) is not None
    for bad in g["video_bad"]:
        assert O.AxialTopology.from_geometry(g["seq_len"], tuple(bad), lt, lh, lw) is None
    t3 = O.AxialTopology.from_geometry(g["seq_len"], tuple(g["video_ok"]), lt, lh, lw, landmarks=3)
    assert t3.frames == 37 and t3.landmark_frames == GOLD["landmarks"]["3"]
    t1 = O.AxialTopology.from_geometry(g["seq_len"], tuple(g["video_ok"]), lt, lh, lw, landmarks=1)
    assert t1.landmark_frames == GOLD["landmarks"]["1"]
    tall = O.AxialTopology.from_geometry(g["seq_len"], tuple(g["video_ok"]), lt, lh, lw, landmarks=999)
    assert len(tall.landmark_frames) == GOLD["landmarks"]["999_count"]


def test_bulk_mask_matches_pairwise():
    t = _topology(GOLD["fixture"])
    s = t.video_span[1]
    m = t.mask_rows(range(s))
    assert m.dtype == np.float32 and set(np.unique(m)) <= {0.0, np.float32(-1e30)}
    assert all((m[q, k] == 0) == t.allows(q, k) for q in range(s) for k in range(s))


# ------------------------------------------------------------- block mask
SPECS = [
    dict(seq_len=4096, frames=16, height=16, width=16, n_random=2, seed=1),
    dict(seq_len=2000, frames=5, height=20, width=20, n_random=3, seed=9),          # ragged last block
    dict(seq_len=1000 + 640, prefix_len=640, frames=10, height=10, width=10, n_random=1, seed=3),
    dict(seq_len=700 + 100, prefix_len=100, frames=7, height=10, width=10, n_random=50, seed=5),  # straddling
    dict(seq_len=128, frames=1, height=8, width=16, n_random=4),                    # single block
]


@pytest.mark.parametrize("kw", SPECS)
def test_blockmask_c_equals_python_twin(kw):
    s = O.mask_spec(**kw)
    rp, ci = O.blockmask_build(s)
    rp2, ci2 = O.blockmask_build_py(s)
    assert np.array_equal(rp, rp2) and np.array_equal(ci, ci2)
    nb = len(rp) - 1
    for i in range(nb):
        row = ci[rp[i]:rp[i + 1]]
        assert np.all(np.diff(row) > 0), "ascending, distinct"
        assert i in row, "every query block keeps itself"
    npb = -(-s.prefix_len // 128)
    for i in range(npb):
        assert rp[i + 1] - rp[i] == nb, "prefix query blocks are dense"
    for i in range(nb):
        assert set(range(npb)) <= set(ci[rp[i]:rp[i + 1]]), "prefix key blocks always kept"


def test_blockmask_rejects_bad_geometry():
    with pytest.raises(ValueError):
        O.blockmask_build(O.mask_spec(seq_len=4000, frames=16, height=16, width=16))


# -------------------------------------------------------------- attention
def _inputs(S, H, seed=4):
    return [O.fill_normal_bf16((S, H, 128), seed, st) for st in (1, 2, 3)]


def test_full_selection_is_dense():
    """AxialReferenceTests.swift:41-62: keeping every block reproduces dense."""
    S, H = 300, 2
    q, k, v = _inputs(S, H)
    rp, ci = O.blockmask_build(O.mask_spec(seq_len=S, prefix_len=S, frames=0, height=0, width=0))
    got = O.attend_streaming(q, k, v, rp, ci)
    want = O.attend_dense_f64(q, k, v)
    rel = np.sqrt(np.mean((got - want) ** 2)) / np.sqrt(np.mean(want ** 2))
    assert rel < 1e-6


def test_streaming_matches_masked():
    """AxialReferenceTests.swift:64-79: the streaming recurrence equals the
    masked definition, here over a sparse ragged block list."""
    s = O.mask_spec(seq_len=700, frames=7, height=10, width=10, radius_t=0, n_random=1, seed=2)
    rp, ci = O.blockmask_build(s)
    q, k, v = _inputs(700, 2, seed=11)
    got = O.attend_streaming(q, k, v, rp, ci)
    want = O.attend_masked(q, k, v, rp, ci)
    rel = np.sqrt(np.mean((got - want) ** 2)) / np.sqrt(np.mean(want ** 2))
    assert rel < 2e-6


def test_query_block_sampling_is_exact():
    """AxialReferenceTests.swift:81-97 (chunking is exact): computing a
    subset of query blocks gives the same rows as computing all."""
    s = O.mask_spec(seq_len=1000, frames=10, height=10, width=10, n_random=2, seed=3)
    rp, ci = O.blockmask_build(s)
    q, k, v = _inputs(1000, 2, seed=5)
    full = O.attend_streaming(q, k, v, rp, ci)
    part = O.attend_streaming(q, k, v, rp, ci, qblocks=[1, 6])
    for b in (1, 6):
        sl = slice(b * 128, min(1000, (b + 1) * 128))
        assert np.array_equal(full[:, sl], part[:, sl])


# --------------------------------------------------------------- prologue
def test_rmsnorm_matches_float64():
    x = O.fill_normal_bf16((64, 3, 128), 7, 1)
    w = O.fill_normal_bf16((128,), 7, 4, 1.0, 0.02)
    y = O.bf16_to_f32(O.rmsnorm(x, w, 1e-6))
    xf = O.bf16_to_f32(x).astype(np.float64)
    ref = xf / np.sqrt((xf ** 2).mean(-1, keepdims=True) + 1e-6) * O.bf16_to_f32(w)
    ulp = np.abs(y - ref) / (np.abs(ref) + 1e-30)
    assert np.max(ulp) <= 2 ** -8  # within one bf16 rounding


def test_rope_identity_and_rotation():
    S = 50
    pos = np.zeros((S, 3), dtype=np.int32)
    t0 = O.rope_table(pos)
    x = O.fill_normal_bf16((S, 2, 128), 8, 1)
    assert np.array_equal(O.rope(x, t0), x), "angle 0 is the identity"
    pos = np.stack([np.arange(S)] * 3, 1).astype(np.int32)
    tab = O.rope_table(pos)
    y = O.bf16_to_f32(O.rope(x, tab))
    ang = np.concatenate([np.outer(pos[:, a], 1e4 ** (-2.0 * np.arange(d // 2) / d))
                          for a, d in enumerate((32, 48, 48))], axis=1)
    xf = O.bf16_to_f32(x)
    c, s_ = np.cos(ang)[:, None], np.sin(ang)[:, None]
    ra = c * xf[..., :64] - s_ * xf[..., 64:]
    rb = s_ * xf[..., :64] + c * xf[..., 64:]
    ref = np.concatenate([ra, rb], -1)
    assert np.max(np.abs(y - ref)) < 0.06  # bf16 table and per-op rounding
    rel = np.sqrt(np.mean((y - ref) ** 2) / np.mean(ref ** 2))
    assert rel < 1e-2
