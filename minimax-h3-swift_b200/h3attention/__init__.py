"""B200 (sm_100a) H3 block-sparse self-attention, behind the reference's
H3AttentionBackend seam.  All compute runs in libh3cuda.so."""
from ._lib import H3CError, load as load_library
from .backend import (AttentionContext, AttentionRegistry, CUDABackend, H3AttentionBackend, H3Error, Machine,
                      SDPABackend, TokenOrdering, sdpa)
from .blockmask import BlockList, MaskSpec, calibrate
from .runtime import Runtime

__all__ = [
    "AttentionContext", "AttentionRegistry", "BlockList", "CUDABackend", "H3AttentionBackend", "H3CError",
    "H3Error", "Machine", "MaskSpec", "Runtime", "SDPABackend", "TokenOrdering", "calibrate", "load_library", "sdpa",
]
