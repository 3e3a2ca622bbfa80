"""Randomised agreement between independent implementations (CPU, hypothesis).

* Block list: the library's host builder, the C checker and the checker's
  pure-Python twin, on random lattices, prefixes, radii, random-block counts
  and seeds (the integer rule must agree bit for bit everywhere).
* Packed layout: the library's segment table against the checker's
  restatement of PackedLayout, on random renders (text length, frame count,
  keyframes, reference blocks), refusals included.
"""
import numpy as np
import pytest

hyp = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from oracle import oracle as O  # noqa: E402

SETTINGS = settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@st.composite
def mask_specs(draw):
    frames = draw(st.integers(1, 9))
    height = draw(st.integers(1, 40))
    width = draw(st.integers(1, 70))
    prefix = draw(st.integers(0, 700))
    video = frames * height * width
    return dict(seq_len=prefix + video, prefix_len=prefix, frames=frames, height=height, width=width,
                radius_t=draw(st.integers(0, 3)), radius_h=draw(st.integers(0, 3)), radius_w=draw(st.integers(0, 3)),
                n_random=draw(st.integers(0, 12)), seed=draw(st.integers(0, 2 ** 64 - 1)))


@SETTINGS
@given(mask_specs())
def test_blockmask_three_builders_agree(kw):
    from h3attention import BlockList, MaskSpec

    bl = BlockList.build(MaskSpec(**kw))
    spec = O.mask_spec(**kw)
    rp, ci = O.blockmask_build(spec)
    rp2, ci2 = O.blockmask_build_py(spec)
    assert np.array_equal(bl.row_ptr, rp) and np.array_equal(bl.col_idx, ci)
    assert np.array_equal(rp2, rp) and np.array_equal(ci2, ci)
    # structural properties: ascending unique rows, diagonal kept, prefix dense
    nb, npb = len(rp) - 1, -(-kw["prefix_len"] // 128)
    for i in range(nb):
        row = ci[rp[i]:rp[i + 1]]
        assert np.all(np.diff(row) > 0) and i in row
        assert all(j in row for j in range(npb))
        if i < npb:
            assert len(row) == nb


GEOMETRIES = [(864, 480), (480, 864), (720, 720), (256, 256), (1280, 704), (640, 352)]


@st.composite
def renders(draw):
    w, h = draw(st.sampled_from(GEOMETRIES))
    length = draw(st.integers(1, 200))
    g = O.latent_geometry(w, h, length)
    n_kf = draw(st.integers(0, 4))
    # mostly on the timeline, sometimes off it (must be refused by both)
    keyframes = draw(st.lists(st.integers(-2, g["frame_count"] + 1), min_size=n_kf, max_size=n_kf))
    refs = draw(st.lists(st.one_of(
        st.builds(lambda lh, lw: dict(kind="image", latent_h=lh, latent_w=lw), st.integers(1, 40), st.integers(1, 60)),
        st.builds(lambda rt: dict(kind="audio", ref_audio_t=rt), st.integers(0, 50)),
        st.builds(lambda lh, lw, lt, rt: dict(kind="video_audio", latent_h=lh, latent_w=lw, latent_t=lt, ref_audio_t=rt),
                  st.integers(2, 30), st.integers(2, 40), st.integers(1, 8), st.integers(0, 30)),
    ), max_size=3))
    return draw(st.integers(0, 600)), (w, h, length), keyframes, refs


@SETTINGS
@given(renders())
def test_packed_layout_library_equals_checker(render):
    from h3attention.layout import LatentGeometry, LayoutError, PackedLayout, ReferenceBlock

    text, geo, keyframes, refs = render
    try:
        segs, pos = O.packed_layout(text, O.latent_geometry(*geo), keyframes, refs)
        want_error = False
    except O.LayoutError:
        want_error = True
    try:
        lay = PackedLayout(text, LatentGeometry.make(*geo), keyframes, [ReferenceBlock(**r) for r in refs])
        got_error = False
    except LayoutError:
        got_error = True
    assert got_error == want_error
    if not want_error:
        assert lay.segments == segs
        assert lay.total_tokens == len(pos)
        assert np.all(np.isfinite(pos))
