"""C-ABI robustness on the device (B200 only): caller block lists are
validated on request, and a context's workspace may grow while a call that
read the old one is still running on another stream."""
import pytest

pytestmark = pytest.mark.gpu


def _blocks(rp, ci, dev):
    import torch

    return torch.tensor(rp, dtype=torch.int32, device=dev), torch.tensor(ci, dtype=torch.int32, device=dev)


def test_validate_accepts_built_lists(gpu):
    from h3attention import BlockList, MaskSpec, Runtime

    rt = Runtime.get(0)
    for spec in (MaskSpec(seq_len=4096, frames=16, height=16, width=16, n_random=2, seed=1), MaskSpec.dense(1000)):
        rt.validate_blocks(BlockList.build(spec).on(gpu))


@pytest.mark.parametrize("rp,ci,why", [
    ([0, 2, 3, 5], [0, 2, 1, 2, 1], "strictly ascending"),        # row 2 descends
    ([0, 2, 3, 5], [0, 1, 3, 0, 2], "outside [0, n_blocks)"),     # column 3 of 3 blocks
    ([0, 2, 1, 3], [0, 1, 2], "decreasing"),                       # row_ptr goes down
    ([0, 2, 3, 9], [0, 1, 2, 0, 1], "decreasing or outside"),     # row_ptr past nnz
    ([1, 2, 3, 5], [0, 1, 2, 0, 1], "row_ptr[0]"),                # does not start at 0
])
def test_validate_refuses_malformed_lists(gpu, rp, ci, why):
    from h3attention import H3CError, Runtime, _lib

    rt = Runtime.get(0)
    with pytest.raises(H3CError) as ei:
        rt.validate_blocks(_blocks(rp, ci, gpu))
    assert ei.value.status == _lib.H3C_ERR_INVALID_ARGUMENT
    assert why in str(ei.value)


def test_workspace_grows_under_a_call_on_another_stream(gpu):
    """A large fused call on stream A, then at once a larger one on stream B
    of the same context: the growth waits for A's call before freeing the
    old workspace, so A's output is still correct."""
    import torch

    from h3attention import BlockList, MaskSpec, Runtime

    rt = Runtime.get(0)
    rt2_ctx_fresh = Runtime(0)  # a fresh context: its workspace starts empty
    w = torch.ones(128, dtype=torch.bfloat16, device=gpu)
    outs = []
    for S, H in ((16384, 8), (32768, 8)):
        q, k, v = (rt.fill_normal(torch.empty((S, H, 128), dtype=torch.bfloat16, device=gpu), 5, st)
                   for st in (1, 2, 3))
        outs.append((S, H, q, k, v, BlockList.build(MaskSpec.dense(S))))
    sa, sb = torch.cuda.Stream(gpu), torch.cuda.Stream(gpu)
    torch.cuda.synchronize()
    res = []
    for (S, H, q, k, v, bl), st in zip(outs, (sa, sb)):
        o = torch.empty_like(q)
        rt2_ctx_fresh.attn_fwd(q=q, k=k, v=v, out=o, layout="SHD", scale=128 ** -0.5, blocks=bl.on(gpu),
                               q_norm=w, k_norm=w, eps=1e-6, stream=st)
        res.append(o)
    torch.cuda.synchronize()
    for (S, H, q, k, v, bl), o in zip(outs, res):
        want = torch.empty_like(q)
        rt.attn_fwd(q=q, k=k, v=v, out=want, layout="SHD", scale=128 ** -0.5, blocks=bl.on(gpu), q_norm=w,
                    k_norm=w, eps=1e-6)
        torch.cuda.synchronize()
        assert torch.equal(o, want)


def test_device_info_reports_nvlink(gpu):
    """h3c_device_info on a B200: SM count and HBM from CUDA, NVLink links,
    version and NVSwitch links from NVML (read-only), P2P peers with native
    atomics (NVLink, not PCIe) from CUDA.  Printed for the record."""
    import torch

    from h3attention import Runtime

    info = Runtime.get(0).device_info()
    print({k: info[k] for k in ("name", "pci_bus_id", "sm_count", "hbm_bytes", "peer_count", "nvlink_links",
                                "nvlink_version", "nvswitch_links", "nvlink_peer_mask", "native_atomic_peer_mask")})
    assert info["cc_major"] == 10 and info["sm_count"] >= 100
    assert info["pci_bus_id"].count(":") == 2
    assert -1 <= info["nvlink_links"] <= 18
    if info["nvlink_links"] > 0:
        assert info["nvlink_version"] >= 1
        assert 0 <= info["nvswitch_links"] <= info["nvlink_links"]
    n = torch.cuda.device_count()
    assert info["peer_count"] <= n - 1
    # native atomics between peers only over NVLink: a subset of the P2P peers
    assert info["native_atomic_peer_mask"] & ~info["nvlink_peer_mask"] == 0


def test_device_alloc_and_free(gpu):
    """h3c_device_alloc / h3c_device_free (device memory for hosts without a
    CUDA runtime binding): a buffer the kernels can use, freed again."""
    import ctypes as C

    from h3attention import Runtime, _lib

    rt = Runtime.get(0)
    L = _lib.load()
    p = C.c_void_p()
    assert L.h3c_device_alloc(rt.ctx, 1 << 20, C.byref(p)) == _lib.H3C_OK and p.value
    assert L.h3c_device_free(rt.ctx, p) == _lib.H3C_OK
    assert L.h3c_device_free(rt.ctx, None) == _lib.H3C_OK
    q = C.c_void_p(1)
    assert L.h3c_device_alloc(rt.ctx, 0, C.byref(q)) == _lib.H3C_OK and not q.value
