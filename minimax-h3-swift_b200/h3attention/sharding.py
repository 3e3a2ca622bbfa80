"""Multi-GPU layouts of the attention call (one process per GPU).

* Head-sharded: the block list is the same for every head (the reference
  broadcasts its mask over heads, Sources/H3Attention/AxialReference.swift:
  103-107), so heads split across ranks with no exchange at all;
  ``head_range`` gives a rank's contiguous heads and the C ABI takes them as
  ``head_offset/head_count``.
* Sequence-sharded (Ulysses-style, for the longest sequences): each rank
  holds a contiguous, block-aligned slice of the tokens for every head.  One
  all-to-all turns ``[S/P, H, D]`` into ``[S, H/P, D]`` (every token, a
  1/P share of the heads), the rank runs the fused call on its heads, and a
  second all-to-all returns ``[S/P, H, D]``.  The exchange uses
  ``torch.distributed.all_to_all_single`` (NCCL over NVLink on GPUs, gloo on
  CPU in the tests).
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

BLOCK = 128


def head_range(rank: int, world: int, heads: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of the heads of ``rank``; sizes differ by at most one."""
    if not (0 <= rank < world) or heads < 0:
        raise ValueError("bad rank/world/heads")
    base, extra = divmod(heads, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def seq_shard_len(seq_len: int, world: int, block: int = BLOCK) -> int:
    """Tokens per rank in the sequence-sharded layout: the sequence is padded
    to world * a multiple of ``block`` so every shard holds whole blocks."""
    per = -(-seq_len // world)
    return -(-per // block) * block


def seq_range(rank: int, world: int, seq_len: int, block: int = BLOCK) -> Tuple[int, int]:
    """[start, stop) of the valid tokens of ``rank`` (may be empty at the end)."""
    n = seq_shard_len(seq_len, world, block)
    return min(rank * n, seq_len), min((rank + 1) * n, seq_len)


def _exchange_to_heads(x, world, group):
    """[S_r, H, D] (this rank's tokens, all heads) -> [P*S_r, H/P, D] (all tokens, this rank's heads)."""
    import torch
    import torch.distributed as dist

    s_r, h, d = x.shape
    hp = h // world
    send = x.reshape(s_r, world, hp, d).permute(1, 0, 2, 3).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.reshape(world * s_r, hp, d)


def _exchange_to_tokens(y, world, group):
    """[P*S_r, H/P, D] -> [S_r, H, D] (inverse of _exchange_to_heads)."""
    import torch
    import torch.distributed as dist

    s, hp, d = y.shape
    s_r = s // world
    send = y.reshape(world, s_r, hp, d).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 0, 2, 3).reshape(s_r, world * hp, d)


def ulysses_attend(q, k, v, seq_len: int, attend: Callable, group=None):
    """Sequence-sharded attention.

    ``q, k, v``: this rank's ``[S_r, H, D]`` slice, S_r = seq_shard_len(...)
    (rows past the valid tokens are padding).  ``attend(qf, kf, vf)`` runs
    the attention over the full sequence ``[P*S_r, H/P, D]`` of this rank's
    heads (valid tokens: the first ``seq_len``) and returns the same shape.
    Returns this rank's ``[S_r, H, D]`` output slice.  H must be divisible
    by the world size."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if q.shape[1] % world:
        raise ValueError(f"heads ({q.shape[1]}) must be divisible by the world size ({world})")
    if q.shape[0] * world < seq_len:
        raise ValueError("shards do not cover the sequence")
    qf, kf, vf = (_exchange_to_heads(t, world, group) for t in (q, k, v))
    of = attend(qf, kf, vf)
    return _exchange_to_tokens(of, world, group)


def cuda_attend_fn(runtime, blocks, seq_len: int, scale: float, q_norm=None, k_norm=None, eps: float = 1e-6,
                   rope_table=None):
    """The ``attend`` callable for ``ulysses_attend`` on a GPU: the fused
    call of the library on ``[S_pad, H/P, D]`` with ``seq_len`` valid tokens."""
    import torch

    def attend(qf, kf, vf):
        out = torch.empty_like(qf)
        qv, kv, vv, ov = (t[:seq_len] for t in (qf, kf, vf, out))
        runtime.attn_fwd(q=qv, k=kv, v=vv, out=ov, layout="SHD", scale=scale, blocks=blocks, q_norm=q_norm,
                         k_norm=k_norm, eps=eps, rope_table=rope_table)
        return out

    return attend


def max_over_ranks(value: float, group=None, device: Optional[object] = None) -> float:
    """The maximum of a per-rank float (timings are reported as the max over ranks)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
