"""Plain-PyTorch fp32 restatement of the attention call, used only as a
checker (bench.py's sampled parity leg, the tests); never on the product path.

It follows the same reference lines as the CPU oracle and works on any torch
device, so a multi-GPU bench run can check its own output at full size on
the GPU after the timed region:

* ``prologue``: H3RMSNorm (Sources/H3Modules/Modulation.swift:116-120) with
  fp32 arithmetic and a bf16 result, then SplitHalfRoPE
  (Sources/H3Modules/DiTBlock.swift:83-103) with every product and every sum
  rounded to bf16 (Tests/H3ModulesTests/QKFusionMetalFixture.swift:57-69).
* ``attend_blocks``: the masked softmax of AxialReference
  (Sources/H3Attention/AxialReference.swift:89-114) restricted to the kept
  128x128 blocks of the sampled query blocks, in fp32; a row with no kept key
  block gives zeros (O / max(l, 1e-30) with l = 0).
"""
from __future__ import annotations

from typing import Iterable, Optional

BLOCK = 128


def _rbf(x):
    import torch

    return x.to(torch.bfloat16).float()


def prologue(x, w, eps: float, table: Optional[object]):
    """x: bf16 [S, H, D]; w: bf16 [D]; table: bf16 [S, half, 4] (c, -s, s, c)
    or None.  Returns bf16 [S, H, D]."""
    import torch

    f = x.float()
    inv = 1.0 / torch.sqrt((f * f).sum(-1, keepdim=True) / f.shape[-1] + eps)
    y = _rbf((f * inv) * w.float())
    if table is not None:
        half = table.shape[1]
        t = table.float()[:, None, :, :]                       # [S, 1, half, 4]
        a, b = y[..., :half], y[..., half:2 * half]
        ra = _rbf(_rbf(t[..., 0] * a) + _rbf(t[..., 1] * b))
        rb = _rbf(_rbf(t[..., 2] * a) + _rbf(t[..., 3] * b))
        y = torch.cat([ra, rb, y[..., 2 * half:]], dim=-1)
    return y.to(torch.bfloat16)


def attend_blocks(q, k, v, row_ptr, col_idx, qblocks: Iterable[int], heads: Iterable[int], scale: float):
    """fp32 output rows of the sampled query blocks: dict (head, qblock) ->
    [rows, D].  q/k/v: bf16 [S, H, D] (already normalised); row_ptr/col_idx:
    host int sequences of the block list."""
    import torch

    S = q.shape[0]
    res = {}
    for h in heads:
        for ib in qblocks:
            r0, r1 = ib * BLOCK, min(S, (ib + 1) * BLOCK)
            cols = [int(c) for c in col_idx[int(row_ptr[ib]):int(row_ptr[ib + 1])]]
            qf = q[r0:r1, h].float()
            if not cols:
                res[(h, ib)] = torch.zeros_like(qf)
                continue
            idx = torch.cat([torch.arange(c * BLOCK, min(S, (c + 1) * BLOCK)) for c in cols]).to(q.device)
            kf, vf = k[idx, h].float(), v[idx, h].float()
            s = (qf @ kf.T) * scale
            p = torch.softmax(s, dim=-1)
            res[(h, ib)] = p @ vf
    return res


def sample_blocks(n_blocks: int, count: int, seed: int):
    """A deterministic spread of query blocks: the first, the last and
    ``count - 2`` seeded picks in between."""
    import random

    rng = random.Random(seed)
    picks = {0, n_blocks - 1}
    while len(picks) < min(count, n_blocks):
        picks.add(rng.randrange(n_blocks))
    return sorted(picks)
