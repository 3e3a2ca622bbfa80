"""The packed layout and its position ids, on CPU.

The checker's restatement of PackedLayout (oracle.packed_layout) is pinned
against the known answers of the reference's own tests
(Tests/H3FoundationTests/PackedLayoutTests.swift) and its documented
geometry figures (LatentGeometry.swift:27-28).  The library's segment table
(h3c_packed_layout, host code) must equal the checker's on every case,
refusals included.  The device positions are checked on the GPU
(test_gpu_layout.py)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

G480 = O.latent_geometry(864, 480, 5 * O.FPS)  # PackedLayoutTests.geometry


def cond_times(segs, pos):
    return [pos[a, 0] for a, b, k in segs if k == "cond"]


# ------------------------------------------------ pins from the reference tests
def test_geometry_figures():
    # PackedLayoutTests: 5 s at 24 fps snaps to 124 frames; 405 rows per frame
    assert G480["frame_count"] == 124
    assert (G480["latent_h"] // 2) * (G480["latent_w"] // 2) == 405
    # LatentGeometry.swift:27-28 verified the lattice at these frame counts
    for f in (5, 22, 39, 73, 124, 141, 362):
        assert O.align_frame_count(f) == f
    assert O.align_frame_count(120) == 124 and O.align_frame_count(1) == 5


def test_endpoint_anchors_exact():
    segs, pos = O.packed_layout(52, G480, keyframes=[0])
    assert cond_times(segs, pos) == [52.0]
    segs, pos = O.packed_layout(52, G480, keyframes=[G480["frame_count"] - 1])
    want = 52.0 + O.video_t_span(G480["latent_t"]) - O.FRAME_RESCALE
    assert cond_times(segs, pos) == [want]


def test_span_sum_equals_frame_count():
    for frames in (5, 22, 39, 124, 175, 362):
        g = O.latent_geometry(864, 480, frames)
        covered = sum(O.FRAMES_PER_TOKEN[k % 5] for k in range(g["latent_t"]))
        assert covered == frames
        general = 52.0 + O.FRAME_RESCALE * (frames - 1)
        reference = 52.0 + O.video_t_span(g["latent_t"]) - O.FRAME_RESCALE
        assert abs(general - reference) < 1e-9


def test_middle_anchor_ordered_and_video_unmoved():
    segs, pos = O.packed_layout(52, G480, keyframes=[0, 60, G480["frame_count"] - 1])
    t = cond_times(segs, pos)
    assert len(t) == 3 and t[0] < t[1] < t[2]
    assert abs(t[1] - (52.0 + O.FRAME_RESCALE * 60.0)) < 1e-9
    assert all(b - a == 405 for a, b, k in segs if k == "cond")
    bare_segs, bare = O.packed_layout(52, G480)
    v0 = [a for a, b, k in segs if k == "video"][0]
    b0 = [a for a, b, k in bare_segs if k == "video"][0]
    assert pos[v0, 0] == bare[b0, 0]


def test_one_anchor_per_second_uniform():
    g = O.latent_geometry(864, 480, 362)
    assert g["frame_count"] == 362
    anchors = list(range(0, g["frame_count"], O.FPS))
    assert len(anchors) == 16
    t = cond_times(*O.packed_layout(52, g, keyframes=anchors))
    gaps = np.diff(t)
    assert np.all(np.abs(gaps - O.FRAME_RESCALE * O.FPS) < 1e-9)


def test_refusals():
    for bad in (-1, G480["frame_count"]):
        with pytest.raises(O.LayoutError):
            O.packed_layout(52, G480, keyframes=[bad])
    with pytest.raises(O.LayoutError):
        O.position_axis(1, 2, 10.0)
    O.position_axis(2, 2, 10.0)


def test_segment_order():
    segs, _ = O.packed_layout(52, G480, refs=[dict(kind="image", latent_h=30, latent_w=54)])
    kinds = [k for _, _, k in segs]
    assert kinds[0] == "text" and kinds[-2:] == ["audio", "video"] and "ref_img" in kinds


# -------------------------------------------------- library vs checker (host)
REF_SETS = [
    [],
    [dict(kind="image", latent_h=30, latent_w=54)],
    [dict(kind="audio", ref_audio_t=17)],
    [dict(kind="audio", ref_audio_t=0)],
    [dict(kind="video", latent_h=20, latent_w=36, latent_t=7, ref_audio_t=0)],
    [dict(kind="video_audio", latent_h=20, latent_w=36, latent_t=3, ref_audio_t=40),
     dict(kind="image", latent_h=16, latent_w=16)],
]
LAYOUT_CASES = [
    (332, (864, 480, 120), [], 0),
    (52, (864, 480, 120), [0, 60, 123], 0),
    (52, (864, 480, 362), list(range(0, 362, 24)), 0),
    (7, (720, 720, 22), [], 1),
    (0, (256, 256, 5), [4], 2),
    (64, (1280, 704, 39), [0], 3),
    (13, (480, 864, 73), [10], 4),
    (100, (864, 480, 124), [], 5),
]


def _library_layout(text, geo, keyframes, refs):
    from h3attention.layout import LatentGeometry, PackedLayout, ReferenceBlock

    g = LatentGeometry.make(*geo)
    return PackedLayout(text, g, keyframes, [ReferenceBlock(**r) for r in refs])


@pytest.mark.parametrize("text,geo,kf,ri", LAYOUT_CASES)
def test_library_segments_equal_checker(text, geo, kf, ri):
    g = O.latent_geometry(*geo)
    from h3attention.layout import LatentGeometry

    lg = LatentGeometry.make(*geo)
    assert (lg.frame_count, lg.latent_t, lg.audio_t, lg.latent_h, lg.latent_w) == (
        g["frame_count"], g["latent_t"], g["audio_t"], g["latent_h"], g["latent_w"])
    segs, pos = O.packed_layout(text, g, kf, REF_SETS[ri])
    lay = _library_layout(text, geo, kf, REF_SETS[ri])
    assert lay.segments == segs
    assert lay.total_tokens == pos.shape[0] == segs[-1][1]
    assert lg.video_tokens == segs[-1][1] - segs[-1][0]
    assert lg.audio_tokens == segs[-2][1] - segs[-2][0]


def test_library_refusals():
    from h3attention.layout import LayoutError

    for bad in (-1, 124):
        with pytest.raises(LayoutError, match="off the timeline"):
            _library_layout(52, (864, 480, 120), [bad], [])
    with pytest.raises(LayoutError):  # a 1-latent-row reference image is off the patch grid
        _library_layout(52, (864, 480, 120), [], [dict(kind="image", latent_h=1, latent_w=16)])
    with pytest.raises(LayoutError):  # more segments than the device table holds
        _library_layout(52, (864, 480, 120), list(range(40)), [])


def test_capacity_query():
    from h3attention import _lib
    from h3attention.layout import LatentGeometry, PackedLayout

    lay = PackedLayout(52, LatentGeometry.make(864, 480, 120), [0, 123])
    spec = lay.spec()
    n, total = C.c_int32(0), C.c_int64(0)
    small = (_lib.Segment * 2)()
    st = _lib.load().h3c_packed_layout(C.byref(spec), small, 2, C.byref(n), C.byref(total), None, 0)
    assert st == _lib.H3C_ERR_CAPACITY and n.value == 5 and total.value == lay.total_tokens


def test_production_shape():
    """The shape of the reference's published dense SDPA figure: 480x864,
    5 s, 332 text tokens -> S = 15,731 (746 text+audio rows, 37 x 405 video)."""
    segs, pos = O.packed_layout(332, O.latent_geometry(864, 480, 120))
    assert pos.shape == (15731, 3)
    assert segs == [(0, 332, "text"), (332, 746, "audio"), (746, 15731, "video")]
    # table from fp32 positions and a shared inv_freq: half = 48
    inv = (1e4 ** (-np.arange(16, dtype=np.float64) / 16)).astype(np.float32)
    tab = O.rope_table_shared(pos.astype(np.float32), inv)
    assert tab.shape == (15731, 48, 4)
    c, s = O.bf16_to_f32(tab[..., 0]), O.bf16_to_f32(tab[..., 2])
    assert np.all(O.bf16_to_f32(tab[..., 3]) == c) and np.all(O.bf16_to_f32(tab[..., 1]) == -s)
    assert np.abs(c * c + s * s - 1).max() < 1e-2


def test_mask_spec_for_layout():
    """The mask geometry of a render follows from its packed layout: every
    row before the target video is prefix, the video is the token lattice."""
    from h3attention import BlockList, MaskSpec

    lay = _library_layout(332, (864, 480, 120), [0], [])
    spec = MaskSpec.for_layout(lay, radius_h=2, radius_w=2, n_random=4, seed=7)
    assert (spec.seq_len, spec.prefix_len) == (lay.total_tokens, lay.range_of("video")[0])
    assert (spec.frames, spec.height, spec.width) == (37, 15, 27)
    assert spec.prefix_len + spec.frames * spec.height * spec.width == spec.seq_len
    bl = BlockList.build(spec)
    rp, ci = O.blockmask_build(O.mask_spec(**{k: getattr(spec, k) for k in (
        "seq_len", "frames", "height", "width", "prefix_len", "radius_h", "radius_w", "n_random", "seed")}))
    assert np.array_equal(bl.row_ptr, rp) and np.array_equal(bl.col_idx, ci)
    npb = -(-spec.prefix_len // 128)
    for i in range(npb):  # prefix rows are dense
        assert bl.row_ptr[i + 1] - bl.row_ptr[i] == bl.n_blocks
