"""Attention on host-resident tensors, with the copies overlapped.

The reference's seam takes and returns ``[H, S, D]`` arrays (MLX unified
memory on Apple silicon, so there is no copy at all there).  On a discrete
GPU a caller holding the operands in host memory pays PCIe/C2C transfers
that are larger than the attention itself at these sizes (3.8 GB in, 1.3 GB
out at config 2).  ``attend_host`` hides most of that: heads are
independent, so the call is cut into head chunks and chunk c's fused call
runs while chunk c+1 is uploaded and chunk c-1 is downloaded, on three CUDA
streams ordered by events.
"""
from __future__ import annotations

from typing import Optional

from .runtime import Runtime


class HostAttention:
    """Reusable device buffers + streams for ``[H, S, D]`` host operands.

    Host tensors should be pinned (``tensor.pin_memory()``) for the copies to
    be asynchronous.  ``chunk_heads`` heads move and compute per stage."""

    def __init__(self, device: int, heads: int, seq_len: int, chunk_heads: int = 4):
        import torch

        self.dev = torch.device("cuda", device)
        self.rt = Runtime.get(device)
        self.heads, self.seq_len = heads, seq_len
        self.chunk = max(1, min(chunk_heads, heads))
        shape = (heads, seq_len, 128)
        self.q, self.k, self.v, self.o = (torch.empty(shape, dtype=torch.bfloat16, device=self.dev)
                                          for _ in range(4))
        self.s_in = torch.cuda.Stream(self.dev)
        self.s_run = torch.cuda.Stream(self.dev)
        self.s_out = torch.cuda.Stream(self.dev)

    def __call__(self, q_host, k_host, v_host, out_host, blocks, scale: float, q_norm=None, k_norm=None,
                 eps: float = 1e-6, rope_table=None, stream: Optional[object] = None):
        """Runs the fused call over host ``[H, S, D]`` tensors into
        ``out_host``; returns after the last download is enqueued on the
        caller's stream (``stream`` or the current stream)."""
        import torch

        caller = stream if stream is not None else torch.cuda.current_stream(self.dev)
        start = torch.cuda.Event()
        start.record(caller)
        for s_ in (self.s_in, self.s_run, self.s_out):
            s_.wait_event(start)
        done_out = None
        for h0 in range(0, self.heads, self.chunk):
            h1 = min(self.heads, h0 + self.chunk)
            with torch.cuda.stream(self.s_in):
                for d, h in ((self.q, q_host), (self.k, k_host), (self.v, v_host)):
                    d[h0:h1].copy_(h[h0:h1], non_blocking=True)
                up = torch.cuda.Event()
                up.record(self.s_in)
            self.s_run.wait_event(up)
            self.rt.attn_fwd(q=self.q, k=self.k, v=self.v, out=self.o, layout="HSD", scale=scale, blocks=blocks,
                             head_offset=h0, head_count=h1 - h0, q_norm=q_norm, k_norm=k_norm, eps=eps,
                             rope_table=rope_table, stream=self.s_run)
            ran = torch.cuda.Event()
            ran.record(self.s_run)
            self.s_out.wait_event(ran)
            with torch.cuda.stream(self.s_out):
                out_host[h0:h1].copy_(self.o[h0:h1], non_blocking=True)
                done_out = torch.cuda.Event()
                done_out.record(self.s_out)
        caller.wait_event(done_out)
