"""The packed sequence the attention sees, and its RoPE table.

Mirrors the reference's ``LatentGeometry`` (Sources/H3Foundation/
LatentGeometry.swift:12-61), ``ReferenceBlock`` / ``PackedLayout``
(Sources/H3Foundation/PackedSequence.swift:149-299) and the table that
``prepareRender`` builds from the layout's position ids and the checkpoint's
``rope.inv_freq`` (Sources/H3Modules/H3Transformer.swift:263-276).  The
segment table comes from ``h3c_packed_layout``; the fp32 positions and the
bf16 table are evaluated on the device by ``h3c_packed_positions_device`` /
``h3c_rope_table_layout``.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

from . import _lib

FPS, LATENT_FPS, LATTICE, LATTICE_OFFSET, SPATIAL_DOWNSAMPLE = 24, 40, 17, 5, 16
SEGMENT_KINDS = ("text", "cond", "ref_img", "ref_audio", "audio", "video")
REF_KINDS = {"image": 0, "audio": 1, "video": 2, "video_audio": 3}


class LayoutError(ValueError):
    """A layout the reference refuses with H3Error (an anchor off the
    timeline, an axis smaller than the patch)."""


@dataclass(frozen=True)
class LatentGeometry:
    """``LatentGeometry(width:height:length:)``: frame count snapped onto
    the 17k+5 lattice, latent_t = 5(F-5)/17 + 2, audio_t = round(F/24*40)."""

    frame_count: int
    latent_t: int
    audio_t: int
    latent_h: int
    latent_w: int
    patch: int = 2

    @staticmethod
    def align_frame_count(length: int) -> int:
        n = max(LATTICE_OFFSET, length)
        return LATTICE_OFFSET + math.ceil((n - LATTICE_OFFSET) / LATTICE) * LATTICE

    @classmethod
    def make(cls, width: int, height: int, length: int, patch: int = 2) -> "LatentGeometry":
        f = cls.align_frame_count(length)
        audio_t = int(math.floor(f / FPS * LATENT_FPS + 0.5))  # Swift rounded(): half away from zero
        return cls(f, 5 * (f - LATTICE_OFFSET) // LATTICE + 2, audio_t, height // SPATIAL_DOWNSAMPLE,
                   width // SPATIAL_DOWNSAMPLE, patch)

    @property
    def video_tokens(self) -> int:
        return self.latent_t * (self.latent_h // self.patch) * (self.latent_w // self.patch)

    @property
    def audio_tokens(self) -> int:
        return 2 * self.audio_t


@dataclass(frozen=True)
class ReferenceBlock:
    kind: str  # image | audio | video | video_audio
    latent_h: int = 0
    latent_w: int = 0
    latent_t: int = 0
    ref_audio_t: int = 0


@dataclass
class PackedLayout:
    """``PackedLayout(textTokens:geometry:keyframes:refs:)``: segments in the
    order text | cond/refs | audio | video, and ``total_tokens`` rows."""

    text_tokens: int
    geometry: LatentGeometry
    keyframes: Sequence[int] = ()
    refs: Sequence[ReferenceBlock] = ()
    segments: List[Tuple[int, int, str]] = field(init=False)
    total_tokens: int = field(init=False)

    def __post_init__(self):
        self._keep = []  # ctypes arrays referenced by the spec
        spec = self.spec()
        n_seg, total = C.c_int32(0), C.c_int64(0)
        L = _lib.load()
        err = C.create_string_buffer(256)
        st = L.h3c_packed_layout(C.byref(spec), None, 0, C.byref(n_seg), C.byref(total), err, 256)
        if st == _lib.H3C_ERR_INVALID_ARGUMENT:
            raise LayoutError(err.value.decode())
        _lib.check(st, what="h3c_packed_layout")
        segs = (_lib.Segment * max(1, n_seg.value))()
        _lib.check(L.h3c_packed_layout(C.byref(spec), segs, n_seg.value, C.byref(n_seg), C.byref(total), None, 0),
                   what="h3c_packed_layout")
        self.segments = [(s.start, s.stop, SEGMENT_KINDS[s.kind]) for s in segs[:n_seg.value]]
        self.total_tokens = total.value

    def spec(self) -> _lib.LayoutSpec:
        g = self.geometry
        kf = (C.c_int32 * max(1, len(self.keyframes)))(*self.keyframes)
        refs = (_lib.RefBlock * max(1, len(self.refs)))(
            *[_lib.RefBlock(REF_KINDS[r.kind], r.latent_h, r.latent_w, r.latent_t, r.ref_audio_t) for r in self.refs])
        self._keep = [kf, refs]
        return _lib.LayoutSpec(self.text_tokens, g.frame_count, g.latent_t, g.audio_t, g.latent_h, g.latent_w,
                               g.patch, len(self.keyframes), kf, len(self.refs), refs)

    def range_of(self, kind: str) -> Tuple[int, int]:
        for a, b, k in self.segments:
            if k == kind:
                return a, b
        raise KeyError(kind)

    def positions(self, device: int = 0, stream=None):
        """fp32 [S, 3] position ids on ``cuda:device`` (Float(positionIds))."""
        import torch

        from .runtime import Runtime, _stream_ptr

        rt = Runtime.get(device)
        out = torch.empty((self.total_tokens, 3), dtype=torch.float32, device=f"cuda:{device}")
        spec = self.spec()
        rt._check(rt.L.h3c_packed_positions_device(rt.ctx, C.byref(spec), out.data_ptr(), self.total_tokens,
                                                   _stream_ptr(stream)))
        return out

    def rope_table(self, inv_freq, device: int = 0, stream=None):
        """bf16 [S, 3n, 4] rotation table from the shared ``inv_freq`` [n]."""
        import torch

        from .runtime import Runtime, _stream_ptr

        rt = Runtime.get(device)
        inv = inv_freq.to(device=f"cuda:{device}", dtype=torch.float32).contiguous()
        n = inv.shape[0]
        out = torch.empty((self.total_tokens, 3 * n, 4), dtype=torch.bfloat16, device=f"cuda:{device}")
        spec = self.spec()
        rt._check(rt.L.h3c_rope_table_layout(rt.ctx, C.byref(spec), inv.data_ptr(), n, out.data_ptr(),
                                             self.total_tokens, _stream_ptr(stream)))
        return out
