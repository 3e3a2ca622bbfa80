"""Per-device handle on the C ABI: one ``h3c_ctx`` per CUDA device.

Torch tensors are accepted for convenience; only their device pointers,
shapes and strides cross the boundary.
"""
from __future__ import annotations

import ctypes as C
import threading
from typing import Dict, Optional

from . import _lib


def _stream_ptr(stream) -> Optional[int]:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None


def view_of(t, layout: str) -> _lib.View:
    """h3c_view of a bf16 tensor.  layout "SHD": [S, H, 128]; "HSD": [H, S, 128]."""
    if t.stride(-1) != 1:
        raise ValueError("head_dim must be contiguous")
    if layout == "SHD":
        tok, head = t.stride(0), t.stride(1)
    elif layout == "HSD":
        head, tok = t.stride(0), t.stride(1)
    else:
        raise ValueError(layout)
    return _lib.View(t.data_ptr(), tok, head)


class Runtime:
    _lock = threading.Lock()
    _by_device: Dict[int, "Runtime"] = {}

    def __init__(self, device: int):
        self.L = _lib.load()
        self.device = device
        h = C.c_void_p()
        _lib.check(self.L.h3c_init(device, C.byref(h)), what=f"h3c_init(device={device})")
        self.ctx = h

    @classmethod
    def get(cls, device: Optional[int] = None) -> "Runtime":
        if device is None:
            import torch

            device = torch.cuda.current_device()
        with cls._lock:
            rt = cls._by_device.get(device)
            if rt is None:
                rt = cls._by_device[device] = Runtime(device)
            return rt

    @staticmethod
    def device_count() -> int:
        n = C.c_int(0)
        _lib.load().h3c_device_count(C.byref(n))
        return n.value

    def _check(self, st: int):
        _lib.check(st, self.ctx)

    def device_info(self) -> dict:
        info = _lib.DevInfo()
        self._check(self.L.h3c_device_info(self.ctx, C.byref(info)))
        d = {f: getattr(info, f) for f, _ in _lib.DevInfo._fields_}
        d["name"] = info.name.decode()
        d["pci_bus_id"] = info.pci_bus_id.decode()
        return d

    # ------------------------------------------------------------ attention
    def attn_args(self, q, k, v, out, layout, scale, blocks, flags=0, heads=None, head_offset=0,
                  head_count=None, q_norm=None, k_norm=None, eps=1e-6, rope_table=None):
        seq_axis = 0 if layout == "SHD" else 1
        head_axis = 1 - seq_axis
        H = q.shape[head_axis] if heads is None else heads
        a = _lib.AttnArgs()
        a.q, a.k, a.v, a.out = (view_of(t, layout) for t in (q, k, v, out))
        a.seq_len = q.shape[seq_axis]
        a.heads = H
        a.head_dim = q.shape[-1]
        a.head_offset = head_offset
        a.head_count = H - head_offset if head_count is None else head_count
        a.scale = scale
        rp, ci = blocks
        a.row_ptr, a.col_idx = rp.data_ptr(), ci.data_ptr()
        a.block = 128
        a.flags = flags
        if q_norm is not None:
            a.flags |= _lib.H3C_FUSE_PROLOGUE
            a.q_norm_weight, a.k_norm_weight = q_norm.data_ptr(), k_norm.data_ptr()
            a.eps = eps
            if rope_table is None:
                a.flags |= _lib.H3C_NO_ROPE
            else:
                a.rope_table = rope_table.data_ptr()
                a.rope_half = rope_table.shape[1]
        return a

    def attn_fwd(self, *, stream=None, **kw):
        a = self.attn_args(**kw)
        self._check(self.L.h3c_attn_fwd(self.ctx, C.byref(a), _stream_ptr(stream)))

    def attn_fwd_sync(self, *, stream=None, **kw):
        """attn_fwd, synchronise, and raise H3CError(H3C_ERR_TIMEOUT) if a
        bounded device wait gave up."""
        a = self.attn_args(**kw)
        self._check(self.L.h3c_attn_fwd_sync(self.ctx, C.byref(a), _stream_ptr(stream)))

    # ------------------------------------------------- sequence-sharded path
    @staticmethod
    def comm_unique_id() -> bytes:
        cid = _lib.CommId()
        _lib.check(_lib.load().h3c_comm_unique_id(C.byref(cid)), what="h3c_comm_unique_id")
        return C.string_at(C.addressof(cid), 128)  # all 128 bytes (the id holds NULs)

    def comm_init(self, unique_id: bytes, nranks: int, rank: int):
        if len(unique_id) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        cid = _lib.CommId()
        C.memmove(C.addressof(cid), unique_id, 128)
        self._check(self.L.h3c_comm_init(self.ctx, C.byref(cid), nranks, rank))

    def attn_fwd_seqshard(self, *, stream=None, timeout_ms=None, **kw):
        """This rank's [S_r, H, D] shards in and out; ``seq_len`` is global.
        With ``timeout_ms`` the call also waits (bounded) for the exchange:
        a rank that does not take part raises H3CError(H3C_ERR_TIMEOUT) after
        the communicator is aborted, instead of hanging."""
        seq_len = kw.pop("seq_len")
        a = self.attn_args(**kw)
        a.seq_len = seq_len
        self._check(self.L.h3c_attn_fwd_seqshard(self.ctx, C.byref(a), _stream_ptr(stream)))
        if timeout_ms is not None:
            self.comm_wait(stream, timeout_ms)

    def comm_wait(self, stream=None, timeout_ms: int = 60000):
        self._check(self.L.h3c_comm_wait(self.ctx, _stream_ptr(stream), int(timeout_ms)))

    def comm_destroy(self):
        self._check(self.L.h3c_comm_destroy(self.ctx))

    def device_status(self):
        self._check(self.L.h3c_device_status(self.ctx))

    def attn_fwd_args(self, a: _lib.AttnArgs, stream=None):
        self._check(self.L.h3c_attn_fwd(self.ctx, C.byref(a), _stream_ptr(stream)))

    # ------------------------------------------------------------- prologue
    def prologue(self, x, out, weight, eps, rope_table=None, layout="SHD", stream=None):
        seq_axis = 0 if layout == "SHD" else 1
        S, H = x.shape[seq_axis], x.shape[1 - seq_axis]
        half = rope_table.shape[1] if rope_table is not None else 0
        self._check(self.L.h3c_prologue(self.ctx, view_of(x, layout), view_of(out, layout), S, H, 0, H,
                                        weight.data_ptr(), eps,
                                        rope_table.data_ptr() if rope_table is not None else None, half,
                                        _stream_ptr(stream)))

    def rope_table(self, pos, dims=(32, 48, 48), theta=1e4, stream=None):
        import torch

        S = pos.shape[0]
        half = sum(dims) // 2
        out = torch.empty((S, half, 4), dtype=torch.bfloat16, device=pos.device)
        d = (C.c_int32 * 3)(*dims)
        self._check(self.L.h3c_rope_table(self.ctx, pos.data_ptr(), S, d, theta, out.data_ptr(),
                                          _stream_ptr(stream)))
        return out

    def rope_table_shared(self, pos, inv_freq, stream=None):
        """The production table: float positions [S, 3] and the shared
        inv_freq [n] (both fp32 on this device); returns bf16 [S, 3n, 4]."""
        import torch

        pos = pos.to(torch.float32).contiguous()
        inv = inv_freq.to(device=pos.device, dtype=torch.float32).contiguous()
        S, n = pos.shape[0], inv.shape[0]
        out = torch.empty((S, 3 * n, 4), dtype=torch.bfloat16, device=pos.device)
        self._check(self.L.h3c_rope_table_shared(self.ctx, pos.data_ptr(), S, inv.data_ptr(), n, out.data_ptr(),
                                                 _stream_ptr(stream)))
        return out

    def fill_normal(self, out, seed, stream_id, mean=0.0, std=1.0, stream=None):
        self._check(self.L.h3c_fill_normal_bf16(self.ctx, out.data_ptr(), out.numel(), seed, stream_id, mean, std,
                                                _stream_ptr(stream)))
        return out

    def validate_blocks(self, blocks, stream=None):
        """Check a device block list (row_ptr [n_blocks+1], col_idx [nnz]
        int32 tensors on this device): row_ptr starts at 0, never decreases
        and ends at nnz; columns in [0, n_blocks), strictly ascending per
        row.  Raises H3CError(H3C_ERR_INVALID_ARGUMENT) with the reason.
        Synchronises the stream."""
        rp, ci = blocks
        self._check(self.L.h3c_blockmask_validate(self.ctx, rp.data_ptr(), ci.data_ptr(), rp.numel() - 1, ci.numel(),
                                                  _stream_ptr(stream)))

    def blockmask_device(self, spec, capacity: int, stream=None):
        import torch

        nb = spec.n_blocks
        rp = torch.empty(nb + 1, dtype=torch.int32, device=f"cuda:{self.device}")
        ci = torch.empty(max(capacity, 1), dtype=torch.int32, device=f"cuda:{self.device}")
        nnz = C.c_int64(0)
        cs = spec.to_c()
        self._check(self.L.h3c_blockmask_build_device(self.ctx, C.byref(cs), rp.data_ptr(), ci.data_ptr(), ci.numel(),
                                                      C.byref(nnz), _stream_ptr(stream)))
        return rp, ci[: nnz.value]
