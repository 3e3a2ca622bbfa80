"""The compacted 128x128 block list (CSR) and its specification.

The reference has no block-sparse mask; this is the new component the
benchmark defines (3D-local window + seed-random key blocks), with
AxialTopology's prefix rule lifted to blocks
(Sources/H3Attention/AxialTopology.swift:128-137): a query block touching the
conditioning prefix keeps every key block, and every query block keeps the
prefix key blocks.  The rule itself is implemented once in C
(``h3c_blockmask_build``) with a bit-identical device twin
(``h3c_blockmask_build_device``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace
from typing import Dict, Optional, Tuple

import numpy as np

from . import _lib

BLOCK = 128


@dataclass(frozen=True)
class MaskSpec:
    """Mirror of h3c_mask_spec.  Tokens [0, prefix_len) are conditioning
    (dense rows and columns); the rest is a frames x height x width lattice
    in t-major, h, w raster order."""

    seq_len: int
    frames: int
    height: int
    width: int
    prefix_len: int = 0
    radius_t: int = 1
    radius_h: int = 1
    radius_w: int = 1
    n_random: int = 0
    seed: int = 0
    cell_t: int = 1
    cell_h: int = 16
    cell_w: int = 32
    block: int = BLOCK

    @property
    def n_blocks(self) -> int:
        return -(-self.seq_len // self.block)

    def to_c(self) -> _lib.MaskSpec:
        s = _lib.MaskSpec()
        for name, _ in _lib.MaskSpec._fields_:
            setattr(s, name, int(getattr(self, name)))
        return s

    @staticmethod
    def for_layout(layout, **params) -> "MaskSpec":
        """The mask of a render's packed sequence (``layout.PackedLayout``):
        every row before the target video (text, conditions, references,
        audio) is prefix, the video is the latent_t x (latent_h/patch) x
        (latent_w/patch) token lattice.  ``params``: radius_*, n_random,
        seed, cell_*."""
        g = layout.geometry
        v0, v1 = layout.range_of("video")
        assert v1 == layout.total_tokens, "the target video is the last segment"
        return MaskSpec(seq_len=layout.total_tokens, frames=g.latent_t, height=g.latent_h // g.patch,
                        width=g.latent_w // g.patch, prefix_len=v0, **params)

    @staticmethod
    def dense(seq_len: int) -> "MaskSpec":
        """Every block kept: the whole sequence is prefix."""
        return MaskSpec(seq_len=seq_len, frames=0, height=0, width=0, prefix_len=seq_len)


@dataclass
class BlockList:
    """CSR block mask: ``row_ptr`` [n_blocks+1], ``col_idx`` [nnz] int32,
    ascending within each row; host copies plus per-device copies."""

    seq_len: int
    row_ptr: np.ndarray
    col_idx: np.ndarray
    block: int = BLOCK
    _dev: Dict[int, Tuple[object, object]] = field(default_factory=dict, repr=False)

    @property
    def n_blocks(self) -> int:
        return len(self.row_ptr) - 1

    @property
    def nnz(self) -> int:
        return int(self.row_ptr[-1])

    @property
    def block_density(self) -> float:
        return self.nnz / float(self.n_blocks * self.n_blocks)

    def kept_pairs(self) -> float:
        """Sum over kept block pairs of valid rows x valid columns."""
        nb = self.n_blocks
        sizes = np.minimum(self.block, self.seq_len - np.arange(nb) * self.block).astype(np.float64)
        rows = np.repeat(sizes, np.diff(self.row_ptr))
        return float(np.sum(rows * sizes[self.col_idx]))

    @property
    def density(self) -> float:
        """Token-pair density over the valid S x S attention."""
        return self.kept_pairs() / float(self.seq_len) ** 2

    def flops(self, heads: int, head_dim: int = 128) -> float:
        """Algorithmic FLOPs of one forward: 4 * H * D * kept pairs (the
        reference counts 4*H*S^2*D for dense attention,
        Tests/H3ModulesTests/HardwareCeilingTests.swift:428-430)."""
        return 4.0 * heads * head_dim * self.kept_pairs()

    @staticmethod
    def build(spec: MaskSpec) -> "BlockList":
        L = _lib.load()
        cs = spec.to_c()
        nnz = C.c_int64(0)
        _lib.check(L.h3c_blockmask_build(C.byref(cs), None, None, 0, C.byref(nnz)), what="h3c_blockmask_build")
        rp = np.empty(spec.n_blocks + 1, dtype=np.int32)
        ci = np.empty(max(nnz.value, 1), dtype=np.int32)
        _lib.check(L.h3c_blockmask_build(C.byref(cs), rp.ctypes.data_as(C.c_void_p), ci.ctypes.data_as(C.c_void_p),
                                         ci.size, C.byref(nnz)), what="h3c_blockmask_build")
        return BlockList(spec.seq_len, rp, ci[: nnz.value], spec.block)

    @staticmethod
    def dense(seq_len: int) -> "BlockList":
        return BlockList.build(MaskSpec.dense(seq_len))

    def on(self, device) -> Tuple[object, object]:
        """Device copies (torch int32 tensors) of row_ptr and col_idx."""
        import torch

        dev = torch.device(device)
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        if idx not in self._dev:
            self._dev[idx] = (torch.from_numpy(self.row_ptr).to(dev), torch.from_numpy(self.col_idx).to(dev))
        return self._dev[idx]


def calibrate(spec: MaskSpec, target: float, radii_t=range(0, 16), n_random=range(0, 121, 2),
              build=None) -> Tuple[MaskSpec, float]:
    """Choose (radius_t, n_random) whose token density is closest to target;
    returns the spec and the measured density (reported, never assumed).
    ``build`` (spec -> BlockList) defaults to the library's builder."""
    build = build or BlockList.build
    best: Optional[Tuple[float, MaskSpec, float]] = None
    for rt in radii_t:
        base = replace(spec, radius_t=rt, n_random=0)
        d0 = build(base).density
        if d0 > target + 0.02 and best is not None:
            break
        for nr in n_random:
            cand = replace(base, n_random=nr)
            d = build(cand).density
            err = abs(d - target)
            if best is None or err < best[0]:
                best = (err, cand, d)
            if d > target:
                break
    assert best is not None
    return best[1], best[2]
