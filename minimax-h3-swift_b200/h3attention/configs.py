"""The benchmark workloads of the H3 attention path (seeded, synthetic).

Each config gives the lattice, heads, mask parameters and RoPE positions.
Inputs are N(0,1) bf16 from the counter-based generator (h3c_fill_normal_bf16),
norm weights 1 + 0.02 N(0,1), eps 1e-6, RoPE theta 1e4 with t/h/w rotary
dims 32/48/48 (64 rotated pairs, so rot == head_dim).
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional, Tuple

import numpy as np

from .blockmask import MaskSpec

ROPE_DIMS = (32, 48, 48)
ROPE_THETA = 1e4
EPS = 1e-6
HEAD_DIM = 128

# generator stream ids
STREAM_Q, STREAM_K, STREAM_V, STREAM_WQ, STREAM_WK = 1, 2, 3, 4, 5


@dataclass(frozen=True)
class Workload:
    name: str
    heads: int
    frames: int
    height: int
    width: int
    audio: int = 0          # 1D-RoPE conditioning tokens placed before the video
    radius_t: int = 1
    radius_h: int = 1
    radius_w: int = 1
    n_random: int = 0
    dense: bool = False
    seed: int = 20260101
    target_density: Optional[float] = None
    eps: float = EPS
    # (text_tokens, width, height, length): positions and RoPE table of the
    # production model, from the packed layout of that render and a shared
    # 16-entry inv_freq (rot 96); None: the benchmark's integer grid table
    render: Optional[Tuple[int, int, int, int]] = None

    @property
    def video_tokens(self) -> int:
        return self.frames * self.height * self.width

    @property
    def seq_len(self) -> int:
        return self.audio + self.video_tokens

    def mask_spec(self) -> MaskSpec:
        if self.dense:
            return MaskSpec.dense(self.seq_len)
        return MaskSpec(seq_len=self.seq_len, frames=self.frames, height=self.height, width=self.width,
                        prefix_len=self.audio, radius_t=self.radius_t, radius_h=self.radius_h,
                        radius_w=self.radius_w, n_random=self.n_random, seed=self.seed)

    def positions(self) -> np.ndarray:
        """int32 [S, 3]: audio tokens (i, 0, 0), then video (t, h, w) raster."""
        t, h, w = np.meshgrid(np.arange(self.frames), np.arange(self.height), np.arange(self.width), indexing="ij")
        vid = np.stack([t.ravel(), h.ravel(), w.ravel()], axis=1)
        if self.audio:
            aud = np.stack([np.arange(self.audio), np.zeros(self.audio, int), np.zeros(self.audio, int)], axis=1)
            vid = np.concatenate([aud, vid], axis=0)
        return np.ascontiguousarray(vid, dtype=np.int32)

    @property
    def rope_half(self) -> int:
        return 3 * len(shared_inv_freq()) if self.render else sum(ROPE_DIMS) // 2

    def packed_layout(self):
        from .layout import LatentGeometry, PackedLayout

        text, width, height, length = self.render
        return PackedLayout(text, LatentGeometry.make(width, height, length))

    def rope_table(self, runtime, device):
        """bf16 [S, rope_half, 4] table on ``device``."""
        import torch

        if self.render:
            lay = self.packed_layout()
            assert lay.total_tokens == self.seq_len, (lay.total_tokens, self.seq_len)
            return lay.rope_table(torch.from_numpy(shared_inv_freq()), torch.device(device).index or 0)
        return runtime.rope_table(torch.from_numpy(self.positions()).to(device), ROPE_DIMS, ROPE_THETA)

    def scaled(self, frames: int, height: int, width: int, heads: Optional[int] = None) -> "Workload":
        return replace(self, frames=frames, height=height, width=width, heads=heads or self.heads)


CONFIGS = {
    # 1: 16^3 grid, 8 heads, +-1 local + 2 random (about 24% of blocks)
    "config1": Workload("config1", heads=8, frames=16, height=16, width=16, n_random=2),
    # 2: 5 s 1344x768 clip, 40 heads, +-1 t / +-2 h,w + 4 random (about 10%)
    "config2": Workload("config2", heads=40, frames=31, height=48, width=84, radius_h=2, radius_w=2, n_random=4),
    # 3: config 2 + 640 audio tokens before the video, audio rows/cols dense
    "config3": Workload("config3", heads=40, frames=31, height=48, width=84, audio=640, radius_h=2, radius_w=2,
                        n_random=4),
    # 4: dense roofline, 32^3
    "config4": Workload("config4", heads=40, frames=32, height=32, width=32, dense=True),
}


def shared_inv_freq(n: int = 16, theta: float = ROPE_THETA) -> np.ndarray:
    """Stand-in for the checkpoint's ``rope.inv_freq`` [16] (no checkpoint
    here): theta^(-k/16), fp32."""
    return (theta ** (-np.arange(n, dtype=np.float64) / n)).astype(np.float32)


# The production model's own call: 480x864, 5 s (124 frames: 37 latent
# frames of 15 x 27 tokens), 332 text tokens + 414 audio rows before the
# video, 56 heads, all blocks kept (the reference runs dense SDPA here),
# eps 1e-5 (H3Config.swift:32), RoPE from the packed layout (rot 96).
CONFIGS["production"] = Workload("production", heads=56, frames=37, height=15, width=27, audio=746, dense=True,
                                 eps=1e-5, render=(332, 864, 480, 120))


def config5(density: float, build=None) -> Workload:
    """864x480 7 s clip, 40 heads; (radius_t, n_random) calibrated per density
    (``build``: the block-list builder used for the calibration)."""
    from .blockmask import calibrate

    base = Workload(f"config5@{density:g}", heads=40, frames=43, height=30, width=54, radius_h=2,
                    radius_w=2, target_density=density)
    spec, _ = calibrate(base.mask_spec(), density, build=build)
    return replace(base, radius_t=spec.radius_t, n_random=spec.n_random)
