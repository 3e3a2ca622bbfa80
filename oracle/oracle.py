"""ctypes front end of the CPU parity checker (``libh3oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``.  The
product (``minimax-h3-swift_b200``) never imports this module.

Each wrapper names the reference function it restates (paths inside the
MiniMax-H3-Swift project).  ``blockmask_build_py`` is a pure-Python twin of the
C mask builder so that the integer generator is pinned by two independent
implementations; ``AxialTopology`` restates the reference's per-token
topology so that its known-answer tests (landmarks, spot checks, closed-form
density) can pin the mask semantics the block mask inherits.

Parity status: partial (see h3_oracle.c header): MLX's SDPA accumulation
order is not reproducible here; the Swift-level semantics are.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


class MaskSpec(C.Structure):
    """Mirror of ``h3o_mask_spec`` (and of ``h3c_mask_spec`` in include/h3cuda.h)."""

    _fields_ = [
        ("seq_len", C.c_int32), ("block", C.c_int32), ("prefix_len", C.c_int32),
        ("frames", C.c_int32), ("height", C.c_int32), ("width", C.c_int32),
        ("cell_t", C.c_int32), ("cell_h", C.c_int32), ("cell_w", C.c_int32),
        ("radius_t", C.c_int32), ("radius_h", C.c_int32), ("radius_w", C.c_int32),
        ("n_random", C.c_int32), ("seed", C.c_uint64),
    ]


class AttnArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
        ("q_tok", C.c_int64), ("q_head", C.c_int64), ("k_tok", C.c_int64),
        ("k_head", C.c_int64), ("v_tok", C.c_int64), ("v_head", C.c_int64),
        ("out", C.c_void_p), ("out_bf16", C.c_void_p), ("o_tok", C.c_int64), ("o_head", C.c_int64),
        ("seq_len", C.c_int32), ("heads", C.c_int32), ("head_dim", C.c_int32), ("block", C.c_int32),
        ("scale", C.c_float), ("row_ptr", C.c_void_p), ("col_idx", C.c_void_p),
    ]


def lib():
    """Load (building on first use if the sources are present) the oracle."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libh3oracle.so")
        src = os.path.join(_HERE, "h3_oracle.c")
        if not os.path.exists(path) or (os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(path)):
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
        L = C.CDLL(path)
        vp, i32, i64, f32, f64, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_double, C.c_uint64
        L.h3o_fill_normal_bf16.argtypes = [vp, i64, u64, u64, f64, f64]
        L.h3o_rmsnorm_rows.argtypes = [vp, i64, i64, vp, i64, i64, vp, i32, i32, i32, f32]
        L.h3o_rope_rows.argtypes = [vp, i64, i64, vp, i32, i32, i32]
        L.h3o_rope_table.argtypes = [vp, i32, vp, f64, vp]
        L.h3o_rope_table_shared.argtypes = [vp, i32, vp, i32, vp]
        L.h3o_blockmask_build.argtypes = [C.POINTER(MaskSpec), vp, vp, C.POINTER(C.c_int64)]
        L.h3o_blockmask_build.restype = C.c_int
        L.h3o_blockmask_check.argtypes = [C.POINTER(MaskSpec)]
        L.h3o_blockmask_check.restype = C.c_int
        L.h3o_attend_streaming.argtypes = [C.POINTER(AttnArgs), vp, i32, i32, i32]
        L.h3o_attend_masked.argtypes = [C.POINTER(AttnArgs)]
        L.h3o_num_threads.restype = C.c_int
        L.h3o_set_num_threads.argtypes = [C.c_int]
        _LIB = L
    return _LIB


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


# ----------------------------------------------------------------- bf16 utils

def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bits."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def fill_normal_bf16(shape, seed: int, stream: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.uint16)
    lib().h3o_fill_normal_bf16(_p(out), out.size, seed, stream, mean, std)
    return out


# ------------------------------------------------------------- prologue (A2-A4)

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """H3RMSNorm (Sources/H3Modules/Modulation.swift:116-120) over [S,H,D] bf16."""
    S, H, D = x.shape
    x = np.ascontiguousarray(x)
    y = np.empty_like(x)
    lib().h3o_rmsnorm_rows(_p(x), H * D, D, _p(y), H * D, D, _p(np.ascontiguousarray(w)), S, H, D, eps)
    return y


def rope(x: np.ndarray, table: np.ndarray) -> np.ndarray:
    """SplitHalfRoPE (Sources/H3Modules/DiTBlock.swift:83-103), per-op bf16 rounding."""
    S, H, D = x.shape
    half = table.shape[1]
    assert 2 * half <= D
    y = np.array(x, copy=True, order="C")
    lib().h3o_rope_rows(_p(y), H * D, D, _p(np.ascontiguousarray(table)), half, S, H)
    return y


def prologue(x: np.ndarray, w: np.ndarray, eps: float, table: np.ndarray | None) -> np.ndarray:
    """AttentionLayer order (DiTBlock.swift:346-352): RMSNorm, then RoPE."""
    y = rmsnorm(x, w, eps)
    return rope(y, table) if table is not None else y


def rope_table(pos: np.ndarray, dims=(32, 48, 48), theta: float = 1e4) -> np.ndarray:
    """H3RoPE.angles/rotationTable (Sources/H3Modules/H3Transformer.swift:62-78)
    with the per-axis split of the benchmark; pos is int [S,3]."""
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    S = pos.shape[0]
    half = sum(dims) // 2
    d = np.asarray(dims, dtype=np.int32)
    t = np.empty((S, half, 4), dtype=np.uint16)
    lib().h3o_rope_table(_p(pos), S, _p(d), theta, _p(t))
    return t


def rope_table_shared(pos: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    """The production H3RoPE (H3Transformer.swift:62-78): float positions
    [S,3], one shared inv_freq [n] for all three axes; half = 3n."""
    pos = np.ascontiguousarray(pos, dtype=np.float32)
    inv = np.ascontiguousarray(inv_freq, dtype=np.float32)
    S, n = pos.shape[0], inv.shape[0]
    t = np.empty((S, 3 * n, 4), dtype=np.uint16)
    lib().h3o_rope_table_shared(_p(pos), S, _p(inv), n, _p(t))
    return t


# ------------------------------------------------------------ packed layout
# Pure-Python restatement of the position ids of the packed sequence, in
# float64 like the reference (Python floats are IEEE doubles and never
# contract into FMA, so every value is the reference's to the last bit).

FPS, LATENT_FPS, LATTICE, LATTICE_OFFSET, SPATIAL_DOWNSAMPLE = 24, 40, 17, 5, 16  # H3Config.swift:59-80
FRAMES_PER_TOKEN = (1, 4, 4, 4, 4)   # PackedSequence.swift:63
FRAME_RESCALE = 5.0 / 3.0            # PackedSequence.swift:65


class LayoutError(ValueError):
    """What the reference throws as H3Error (keyframeIndex, dimensionOffGrid)."""


def align_frame_count(length: int) -> int:
    """LatentGeometry.alignFrameCount (LatentGeometry.swift:21-25)."""
    import math
    n = max(LATTICE_OFFSET, length)
    k = int(math.ceil(float(n - LATTICE_OFFSET) / float(LATTICE)))
    return LATTICE_OFFSET + k * LATTICE


def latent_geometry(width: int, height: int, length: int) -> dict:
    """LatentGeometry.init (LatentGeometry.swift:29-37); Swift's rounded()
    is half away from zero."""
    import math
    f = align_frame_count(length)
    x = float(f) / float(FPS) * float(LATENT_FPS)
    audio_t = int(math.floor(x + 0.5))
    return dict(frame_count=f, latent_t=5 * (f - LATTICE_OFFSET) // LATTICE + 2, audio_t=audio_t,
                latent_h=height // SPATIAL_DOWNSAMPLE, latent_w=width // SPATIAL_DOWNSAMPLE, patch=2)


def position_axis(dim: int, patch: int, sqrt_area: float):
    """PositionGrid.axis (PackedSequence.swift:69-78)."""
    ratio = float(dim) / sqrt_area
    n = dim // patch
    if n <= 0:
        raise LayoutError(f"dimension {dim} off the patch grid {patch}")
    step = ratio / float(n)
    origin = (1.0 - ratio) / 2.0
    return [(float(i) * step + origin) * 32.0 for i in range(n)]


def frame_grid(h: int, w: int, patch: int = 2):
    """PositionGrid.frameGrid (PackedSequence.swift:82-92)."""
    import math
    area = math.sqrt(float(h) * float(w))
    ha, wa = position_axis(h, patch, area), position_axis(w, patch, area)
    return [(hv, wv) for hv in ha for wv in wa], wa


def video_t_grid(n: int, origin: float):
    """PositionGrid.videoTGrid (PackedSequence.swift:95-103)."""
    out, acc = [], origin
    for k in range(n):
        out.append(acc)
        acc += FRAME_RESCALE * float(FRAMES_PER_TOKEN[k % 5])
    return out


def video_t_span(n: int) -> float:
    """PositionGrid.videoTSpan (PackedSequence.swift:107-109)."""
    acc = 0.0
    for k in range(n):
        acc = acc + FRAME_RESCALE * float(FRAMES_PER_TOKEN[k % 5])
    return acc


def cond_t(text_tokens: int, latent_t: int, frame_count: int, p: int) -> float:
    """PositionGrid.condT (PackedSequence.swift:137-142)."""
    if p == 0:
        return float(text_tokens)
    if p == frame_count - 1:
        return float(text_tokens) + video_t_span(latent_t) - FRAME_RESCALE
    return float(text_tokens) + FRAME_RESCALE * float(p)


SEG_KINDS = ("text", "cond", "ref_img", "ref_audio", "audio", "video")   # SegmentKind order


def packed_layout(text_tokens: int, geometry: dict, keyframes=(), refs=()):
    """PackedLayout.init (PackedSequence.swift:192-297).  ``refs`` entries are
    dicts with kind in (image, audio, video, video_audio), latent_h, latent_w,
    latent_t, ref_audio_t.  Returns (segments [(start, stop, kind)], positions
    as a float64 array [S, 3])."""
    g = geometry
    patch = g.get("patch", 2)
    frame, w_axis = frame_grid(g["latent_h"], g["latent_w"], patch)
    w_low, w_high = w_axis[0], w_axis[-1]
    pos, segs, row = [], [], 0

    def seg(n, kind):
        nonlocal row
        segs.append((row, row + n, kind))
        row += n

    seg(text_tokens, "text")
    pos += [(float(i), 0.0, 0.0) for i in range(text_tokens)]
    cursor = float(text_tokens)
    for p in keyframes:
        if p < 0 or p >= g["frame_count"]:
            raise LayoutError(f"keyframe {p} off the timeline of {g['frame_count']} frames")
        ct = cond_t(text_tokens, g["latent_t"], g["frame_count"], p)
        seg(len(frame), "cond")
        pos += [(ct, h, w) for h, w in frame]
    for b in refs:
        kind = b["kind"]
        if kind == "image":
            rf, _ = frame_grid(b["latent_h"], b["latent_w"], patch)
            seg(len(rf), "ref_img")
            pos += [(cursor, h, w) for h, w in rf]
            cursor += 1.0
        elif kind == "audio":
            rt = b.get("ref_audio_t", 0)
            if rt > 0:
                seg(2 * rt, "ref_audio")
                for w in (w_low, w_high):
                    pos += [(cursor + float(i), 0.0, w) for i in range(rt)]
            cursor += float(rt)
        elif kind in ("video", "video_audio"):
            rt, vt = b.get("ref_audio_t", 0), b["latent_t"]
            rf, rw = frame_grid(b["latent_h"], b["latent_w"], patch)
            if rt > 0:
                seg(2 * rt, "ref_audio")
                for w in (rw[0], rw[-1]):
                    pos += [(cursor + float(i), 0.0, w) for i in range(rt)]
            seg(vt * len(rf), "ref_img")
            for t in video_t_grid(vt, cursor):
                pos += [(t, h, w) for h, w in rf]
            cursor += max(float(rt), video_t_span(vt))
        else:
            raise LayoutError(f"unknown reference kind {kind}")
    seg(2 * g["audio_t"], "audio")
    for w in (w_low, w_high):
        pos += [(cursor + float(i), 0.0, w) for i in range(g["audio_t"])]
    seg(g["latent_t"] * len(frame), "video")
    for t in video_t_grid(g["latent_t"], cursor):
        pos += [(t, h, w) for h, w in frame]
    return segs, np.array(pos, dtype=np.float64).reshape(-1, 3)


# ----------------------------------------------------------------- block mask

def mask_spec(**kw) -> MaskSpec:
    s = MaskSpec()
    defaults = dict(block=128, prefix_len=0, cell_t=1, cell_h=16, cell_w=32,
                    radius_t=1, radius_h=1, radius_w=1, n_random=0, seed=0)
    defaults.update(kw)
    for k, v in defaults.items():
        setattr(s, k, v)
    return s


def blockmask_build(spec: MaskSpec):
    """C builder -> (row_ptr int32[nb+1], col_idx int32[nnz])."""
    L = lib()
    nnz = C.c_int64(0)
    st = L.h3o_blockmask_build(C.byref(spec), None, None, C.byref(nnz))
    if st:
        raise ValueError(f"invalid mask spec (status {st})")
    nb = -(-spec.seq_len // spec.block)
    rp = np.empty(nb + 1, dtype=np.int32)
    ci = np.empty(max(nnz.value, 1), dtype=np.int32)
    L.h3o_blockmask_build(C.byref(spec), _p(rp), _p(ci), C.byref(nnz))
    return rp, ci[: nnz.value]


_M64 = (1 << 64) - 1


def _splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & _M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _M64
    return x ^ (x >> 31)


def blockmask_build_py(spec: MaskSpec):
    """Pure-Python twin of h3o_blockmask_build (same rule, independent code)."""
    S, B, P = spec.seq_len, spec.block, spec.prefix_len
    nb = -(-S // B)
    npb = -(-P // B)
    per = spec.height * spec.width

    def cell(b):
        v = b * B - P
        t, rem = divmod(v, per)
        return t // spec.cell_t, (rem // spec.width) // spec.cell_h, (rem % spec.width) // spec.cell_w

    rows = []
    for i in range(nb):
        if i < npb:
            rows.append(list(range(nb)))
            continue
        keep = set(range(min(npb, nb)))
        qc = cell(i)
        for j in range(npb, nb):
            kc = cell(j)
            if (abs(kc[0] - qc[0]) <= spec.radius_t and abs(kc[1] - qc[1]) <= spec.radius_h
                    and abs(kc[2] - qc[2]) <= spec.radius_w):
                keep.add(j)
        state = (spec.seed ^ ((i * 0x9E3779B97F4A7C15) & _M64)) & _M64
        added = 0
        for _ in range(64 + 16 * spec.n_random):
            if added >= spec.n_random:
                break
            state = _splitmix64(state)
            j = ((state >> 32) * nb) >> 32
            if j not in keep:
                keep.add(j)
                added += 1
        rows.append(sorted(keep))
    rp = np.zeros(nb + 1, dtype=np.int32)
    rp[1:] = np.cumsum([len(r) for r in rows])
    ci = np.array([j for r in rows for j in r], dtype=np.int32)
    return rp, ci


def kept_flops(row_ptr, col_idx, seq_len, heads, head_dim, block=128) -> float:
    """4*H*D*sum over kept block pairs of valid rows x valid cols."""
    nb = len(row_ptr) - 1
    sizes = np.minimum(block, seq_len - np.arange(nb) * block).astype(np.float64)
    counts = np.diff(row_ptr)
    rows = np.repeat(sizes, counts)
    cols = sizes[col_idx]
    return 4.0 * heads * head_dim * float(np.sum(rows * cols))


# ------------------------------------------------------------------ attention

def _attn_args(q, k, v, row_ptr, col_idx, scale, block, out=None, out_bf16=None):
    """q, k, v: [S,H,D] bf16 (uint16) arrays."""
    S, H, D = q.shape
    a = AttnArgs()
    a.q, a.k, a.v = _p(q), _p(k), _p(v)
    a.q_tok = a.k_tok = a.v_tok = H * D
    a.q_head = a.k_head = a.v_head = D
    a.out = _p(out)
    a.out_bf16 = _p(out_bf16)
    a.o_tok, a.o_head = H * D, D
    a.seq_len, a.heads, a.head_dim, a.block = S, H, D, block
    a.scale = scale
    a.row_ptr, a.col_idx = _p(row_ptr), _p(col_idx)
    return a


def attend_streaming(q, k, v, row_ptr, col_idx, scale=None, block=128, qblocks=None, heads=None):
    """AxialReference.attendStreamingKeys (AxialReference.swift:129-171) over the
    kept blocks.  q/k/v [S,H,D] bf16 bits.  Returns fp32 [H,S,D]; rows of query
    blocks not in ``qblocks`` and heads outside ``heads`` stay zero."""
    q, k, v = (np.ascontiguousarray(t) for t in (q, k, v))
    S, H, D = q.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((H, S, D), dtype=np.float32)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    a = _attn_args(q, k, v, rp, ci, scale, block, out=out)
    h0, hn = (0, H) if heads is None else (heads[0], heads[1] - heads[0])
    if qblocks is None:
        lib().h3o_attend_streaming(C.byref(a), None, 0, h0, hn)
    else:
        qb = np.ascontiguousarray(qblocks, dtype=np.int32)
        lib().h3o_attend_streaming(C.byref(a), _p(qb), len(qb), h0, hn)
    return out


def attend_masked(q, k, v, row_ptr, col_idx, scale=None, block=128):
    """AxialReference.attend (AxialReference.swift:89-114): the definition."""
    q, k, v = (np.ascontiguousarray(t) for t in (q, k, v))
    S, H, D = q.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((H, S, D), dtype=np.float32)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    a = _attn_args(q, k, v, rp, ci, scale, block, out=out)
    lib().h3o_attend_masked(C.byref(a))
    return out


def attend_dense_f64(q, k, v, scale=None):
    """Plain dense softmax attention in float64 (numpy), [S,H,D] -> [H,S,D]."""
    qf, kf, vf = (bf16_to_f32(t).astype(np.float64).transpose(1, 0, 2) for t in (q, k, v))
    scale = 1.0 / np.sqrt(qf.shape[-1]) if scale is None else scale
    s = np.einsum("hqd,hkd->hqk", qf, kf) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("hqk,hkd->hqd", p, vf)


# ------------------------------------------- AxialTopology (mask semantics pin)

class AxialTopology:
    """Restatement of Sources/H3Attention/AxialTopology.swift:47-170.

    Only used to pin the prefix rule and the counted-density discipline that
    the block mask inherits, against the reference's own known answers."""

    def __init__(self, sequence_length, video_span, frames, height, width, landmark_frames):
        lo, hi = video_span
        if frames * height * width != hi - lo or hi != sequence_length or lo < 0:
            raise ValueError("geometry does not fill the video span")
        if any(not (0 <= f < frames) for f in landmark_frames):
            raise ValueError("landmark out of range")
        self.prefix = (0, lo)
        self.video_span = (lo, hi)
        self.frames, self.height, self.width = frames, height, width
        self.landmark_frames = sorted(set(landmark_frames))

    @staticmethod
    def from_geometry(sequence_length, video_span, latent_t, latent_h, latent_w, patch=(1, 2, 2),
                      landmarks=3):
        """AxialTopology.swift:82-112."""
        h, w, f = latent_h // patch[1], latent_w // patch[2], latent_t
        lo, hi = video_span
        if f * h * w != hi - lo or hi != sequence_length or lo < 0:
            return None
        n = max(2, min(landmarks, f))
        if n >= f:
            lm = list(range(f))
        else:
            # Swift's .rounded() is round-half-away-from-zero.
            lm = sorted({int(np.floor(i * (f - 1) / (n - 1) + 0.5)) for i in range(n)})
        return AxialTopology(sequence_length, video_span, f, h, w, lm)

    @property
    def tokens_per_frame(self):
        return self.height * self.width

    def locate(self, token):
        lo, hi = self.video_span
        if not (lo <= token < hi):
            return None
        v = token - lo
        per = self.tokens_per_frame
        return v // per, (v % per) // self.width, v % self.width

    def allows(self, query, key):
        if self.prefix[0] <= query < self.prefix[1]:
            return True
        if self.prefix[0] <= key < self.prefix[1]:
            return True
        q, k = self.locate(query), self.locate(key)
        if q is None or k is None:
            return False
        if q[0] == k[0]:
            return True
        if q[1] == k[1] and q[2] == k[2]:
            return True
        return k[0] in self.landmark_frames

    @property
    def density(self):
        s = self.video_span[1]
        p = self.prefix[1] - self.prefix[0]
        per = self.tokens_per_frame
        lms = set(self.landmark_frames)
        video_allowed = 0
        for f0 in range(self.frames):
            full = len(lms) if f0 in lms else len(lms) + 1
            per_query = per * full + (self.frames - full)
            video_allowed += per * (p + per_query)
        return (p * s + video_allowed) / (s * s)

    def mask_rows(self, rows):
        """AxialReference.maskRows (AxialReference.swift:42-84): 0 / -1e30."""
        s = self.video_span[1]
        out = np.full((len(rows), s), -1e30, dtype=np.float32)
        for r, q in enumerate(rows):
            for k in range(s):
                if self.allows(q, k):
                    out[r, k] = 0.0
        return out
