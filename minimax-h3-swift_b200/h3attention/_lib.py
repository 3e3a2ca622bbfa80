"""ctypes binding of ``libh3cuda.so`` (the C ABI declared in include/h3cuda.h).

This is the binding a Python caller of the library uses; the Swift
``CH3Cuda`` module map binds the same header.  Loading fails loudly when the
shared library is missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "libh3cuda.so")

H3C_OK = 0
H3C_ERR_INVALID_ARGUMENT = 1
H3C_ERR_UNSUPPORTED = 2
H3C_ERR_CUDA = 3
H3C_ERR_NCCL = 4
H3C_ERR_TIMEOUT = 5
H3C_ERR_CAPACITY = 6
H3C_ERR_NO_DEVICE = 7

STATUS_NAMES = {
    0: "H3C_OK", 1: "H3C_ERR_INVALID_ARGUMENT", 2: "H3C_ERR_UNSUPPORTED", 3: "H3C_ERR_CUDA",
    4: "H3C_ERR_NCCL", 5: "H3C_ERR_TIMEOUT", 6: "H3C_ERR_CAPACITY", 7: "H3C_ERR_NO_DEVICE",
}

H3C_FUSE_PROLOGUE = 1
H3C_KERNEL_MMA_SYNC = 2
H3C_NO_ROPE = 4

# Every exported symbol of include/h3cuda.h, checked by the CPU test suite.
EXPORTS = (
    "h3c_abi_version", "h3c_init", "h3c_destroy", "h3c_last_error", "h3c_device_info",
    "h3c_device_count", "h3c_blockmask_build", "h3c_blockmask_build_device", "h3c_rope_table",
    "h3c_rope_table_shared", "h3c_packed_layout", "h3c_packed_positions_device", "h3c_rope_table_layout",
    "h3c_prologue", "h3c_attn_fwd", "h3c_attn_workspace_size", "h3c_attn_fwd_sync",
    "h3c_fill_normal_bf16", "h3c_attn_fwd_noalloc", "h3c_device_status",
    "h3c_comm_unique_id", "h3c_comm_init", "h3c_comm_destroy", "h3c_attn_fwd_seqshard",
    "h3c_blockmask_validate", "h3c_attn_fwd_noalloc_status", "h3c_nvlink_query",
    "h3c_device_alloc", "h3c_device_free", "h3c_comm_wait",
)


class H3CError(RuntimeError):
    """A non-zero h3c_status, with the library's message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class DevInfo(C.Structure):
    _fields_ = [
        ("device", C.c_int32), ("cc_major", C.c_int32), ("cc_minor", C.c_int32),
        ("sm_count", C.c_int32), ("hbm_bytes", C.c_int64), ("hbm_free_bytes", C.c_int64),
        ("max_smem_per_block_optin", C.c_int32), ("l2_bytes", C.c_int32),
        ("peer_count", C.c_int32), ("nvlink_peer_mask", C.c_int32), ("name", C.c_char * 96),
        ("nvlink_links", C.c_int32), ("nvlink_version", C.c_int32), ("nvswitch_links", C.c_int32),
        ("native_atomic_peer_mask", C.c_int32), ("pci_bus_id", C.c_char * 16),
    ]


class NvLink(C.Structure):
    _fields_ = [("available", C.c_int32), ("links_active", C.c_int32), ("links_to_switch", C.c_int32),
                ("links_to_gpu", C.c_int32), ("version", C.c_int32)]


class MaskSpec(C.Structure):
    _fields_ = [
        ("seq_len", C.c_int32), ("block", C.c_int32), ("prefix_len", C.c_int32),
        ("frames", C.c_int32), ("height", C.c_int32), ("width", C.c_int32),
        ("cell_t", C.c_int32), ("cell_h", C.c_int32), ("cell_w", C.c_int32),
        ("radius_t", C.c_int32), ("radius_h", C.c_int32), ("radius_w", C.c_int32),
        ("n_random", C.c_int32), ("seed", C.c_uint64),
    ]


class View(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("token_stride", C.c_int64), ("head_stride", C.c_int64)]


class RefBlock(C.Structure):
    _fields_ = [("kind", C.c_int32), ("latent_h", C.c_int32), ("latent_w", C.c_int32), ("latent_t", C.c_int32),
                ("ref_audio_t", C.c_int32)]


class LayoutSpec(C.Structure):
    _fields_ = [
        ("text_tokens", C.c_int32), ("frame_count", C.c_int32), ("latent_t", C.c_int32), ("audio_t", C.c_int32),
        ("latent_h", C.c_int32), ("latent_w", C.c_int32), ("patch", C.c_int32),
        ("n_keyframes", C.c_int32), ("keyframes", C.POINTER(C.c_int32)),
        ("n_refs", C.c_int32), ("refs", C.POINTER(RefBlock)),
    ]


class Segment(C.Structure):
    _fields_ = [("start", C.c_int32), ("stop", C.c_int32), ("kind", C.c_int32)]


class CommId(C.Structure):
    _fields_ = [("internal", C.c_char * 128)]


class AttnArgs(C.Structure):
    _fields_ = [
        ("q", View), ("k", View), ("v", View), ("out", View),
        ("seq_len", C.c_int32), ("heads", C.c_int32), ("head_dim", C.c_int32),
        ("head_offset", C.c_int32), ("head_count", C.c_int32), ("scale", C.c_float),
        ("row_ptr", C.c_void_p), ("col_idx", C.c_void_p), ("block", C.c_int32), ("flags", C.c_int32),
        ("q_norm_weight", C.c_void_p), ("k_norm_weight", C.c_void_p), ("eps", C.c_float),
        ("rope_table", C.c_void_p), ("rope_half", C.c_int32),
    ]


_lock = threading.Lock()
_lib = None


def load() -> C.CDLL:
    """Load libh3cuda.so; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libh3cuda.so not built at {LIB_PATH}; run __graft_entry__.build() or make -C csrc")
        L = C.CDLL(LIB_PATH)
        vp, i32, i64, u64, f32, f64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_double
        st = C.c_int
        sig = {
            "h3c_abi_version": ([], C.c_int),
            "h3c_init": ([C.c_int, C.POINTER(vp)], st),
            "h3c_destroy": ([vp], st),
            "h3c_last_error": ([vp], C.c_char_p),
            "h3c_device_info": ([vp, C.POINTER(DevInfo)], st),
            "h3c_device_count": ([C.POINTER(C.c_int)], st),
            "h3c_blockmask_build": ([C.POINTER(MaskSpec), vp, vp, i64, C.POINTER(i64)], st),
            "h3c_blockmask_build_device": ([vp, C.POINTER(MaskSpec), vp, vp, i64, C.POINTER(i64), vp], st),
            "h3c_rope_table": ([vp, vp, i32, C.POINTER(i32), f64, vp, vp], st),
            "h3c_rope_table_shared": ([vp, vp, i32, vp, i32, vp, vp], st),
            "h3c_packed_layout": ([C.POINTER(LayoutSpec), C.POINTER(Segment), i32, C.POINTER(i32), C.POINTER(i64),
                                   C.c_char_p, C.c_size_t], st),
            "h3c_packed_positions_device": ([vp, C.POINTER(LayoutSpec), vp, i64, vp], st),
            "h3c_rope_table_layout": ([vp, C.POINTER(LayoutSpec), vp, i32, vp, i64, vp], st),
            "h3c_prologue": ([vp, View, View, i32, i32, i32, i32, vp, f32, vp, i32, vp], st),
            "h3c_attn_fwd": ([vp, C.POINTER(AttnArgs), vp], st),
            "h3c_attn_workspace_size": ([C.POINTER(AttnArgs), C.POINTER(C.c_size_t)], st),
            "h3c_attn_fwd_sync": ([vp, C.POINTER(AttnArgs), vp], st),
            "h3c_fill_normal_bf16": ([vp, vp, i64, u64, u64, f64, f64, vp], st),
            "h3c_device_status": ([vp], st),
            "h3c_comm_unique_id": ([C.POINTER(CommId)], st),
            "h3c_comm_init": ([vp, C.POINTER(CommId), C.c_int, C.c_int], st),
            "h3c_comm_destroy": ([vp], st),
            "h3c_attn_fwd_seqshard": ([vp, C.POINTER(AttnArgs), vp], st),
            "h3c_attn_fwd_noalloc": ([C.POINTER(AttnArgs), vp, C.c_char_p, C.c_size_t], st),
            "h3c_attn_fwd_noalloc_status": ([], st),
            "h3c_nvlink_query": ([C.c_char_p, C.POINTER(NvLink)], st),
            "h3c_device_alloc": ([vp, C.c_size_t, C.POINTER(vp)], st),
            "h3c_comm_wait": ([vp, vp, i64], st),
            "h3c_device_free": ([vp, vp], st),
            "h3c_blockmask_validate": ([vp, vp, vp, i32, i64, vp], st),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
        return L


def check(status: int, ctx=None, what: str = "") -> None:
    if status != H3C_OK:
        msg = load().h3c_last_error(ctx).decode() if ctx is not None else what
        raise H3CError(status, msg or what)
