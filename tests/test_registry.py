"""The backend seam's host logic, with the reference's fake backends
(Tests/H3AttentionTests/AttentionRegistryTests.swift:17-37,
Tests/H3ModulesTests/AttentionSeamTests.swift:20-55).  No GPU."""
import pytest

from h3attention import (AttentionContext, AttentionRegistry, CUDABackend, H3AttentionBackend, H3Error, Machine,
                         MaskSpec, SDPABackend, TokenOrdering)

MACHINE = Machine(model="x86_64", chip="test host", memory_bytes=64 << 30, cores=8,
                  cuda_devices=({"cc_major": 10, "cc_minor": 0, "name": "fake B200"},))
NO_GPU = Machine(model="x86_64", chip="cpu only", memory_bytes=64 << 30, cores=8)


class DecliningBackend(H3AttentionBackend):
    identifier = "declining"
    equivalence_class = 0.25
    materialises_scores = False
    prefers_morton_order = True

    @classmethod
    def is_available(cls, machine):
        return True

    def attend(self, queries, keys, values, scale, mask, context):
        return None


class UnavailableBackend(DecliningBackend):
    identifier = "unavailable"
    equivalence_class = 0.5
    prefers_morton_order = False

    @classmethod
    def is_available(cls, machine):
        return False


CTX = AttentionContext(block_index=0, block_count=50, schedule_progress=0.5, sequence_length=4, video_span=None)


def test_backend_is_what_was_named():
    s = AttentionRegistry.resolve("declining", MACHINE, None, [SDPABackend, DecliningBackend])
    assert s.identifier == "declining" and s.equivalence_class == 0.25 and not s.materialises_scores
    assert isinstance(s.backend, DecliningBackend)
    assert s.backend.attend(None, None, None, 1.0, None, CTX) is None


def test_ordering_follows_backend():
    assert AttentionRegistry.resolve("declining", MACHINE, None, [DecliningBackend]).ordering == \
        TokenOrdering.MORTON_PER_FRAME
    assert AttentionRegistry.resolve("sdpa", MACHINE, None, [SDPABackend]).ordering == TokenOrdering.NONE
    assert AttentionRegistry.resolve("declining", MACHINE, TokenOrdering.NONE, [DecliningBackend]).ordering == \
        TokenOrdering.NONE


def test_auto_skips_unavailable():
    s = AttentionRegistry.resolve("auto", MACHINE, None, [UnavailableBackend, DecliningBackend])
    assert s.identifier == "declining"


def test_refuses_rather_than_falls_back():
    with pytest.raises(H3Error):
        AttentionRegistry.resolve("sol", MACHINE, None, [SDPABackend])
    with pytest.raises(H3Error):
        AttentionRegistry.resolve("unavailable", MACHINE, None, [UnavailableBackend])
    with pytest.raises(H3Error):  # no sm_100 device: the CUDA backends are unavailable, never emulated
        AttentionRegistry.resolve("sdpa", NO_GPU)
    with pytest.raises(H3Error):
        AttentionRegistry.resolve("b200-block-sparse", NO_GPU)


def test_cuda_backend_declines_without_prepared_layout():
    b = CUDABackend()
    assert b.attend(None, None, None, 0.1, None, CTX) is None
    b.prepare_render(MaskSpec(seq_len=4096, frames=16, height=16, width=16, n_random=2))
    # non-tensor / wrong-shape operands are declined, not mis-indexed
    assert b.attend(None, None, None, 0.1, None, CTX) is None


def test_registry_lists_both_cuda_backends():
    ids = [t.identifier for t in AttentionRegistry.available]
    assert ids == ["sdpa", "b200-block-sparse"]
