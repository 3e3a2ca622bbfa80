"""The C ABI on CPU: the library loads, exports every declared symbol,
validates arguments, and its host block-mask builder matches the checker
bit for bit.  No GPU compute is called."""
import ctypes as C
import re
import os

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from h3attention import _lib

    return _lib


def test_header_and_exports(lib):
    L = lib.load()
    hdr = open(os.path.join(ROOT, "include", "h3cuda.h")).read()
    declared = set(re.findall(r"\b(h3c_[a-z0-9_]+)\s*\(", hdr))
    assert declared == set(lib.EXPORTS)
    for name in declared:
        assert hasattr(L, name), name
    assert L.h3c_abi_version() == 2


def test_struct_layout_matches_header(lib):
    # sizes computed by the C compiler for the same declarations
    assert C.sizeof(lib.MaskSpec) == 13 * 4 + 4 + 8
    assert C.sizeof(lib.View) == 24
    assert C.sizeof(lib.DevInfo) == 4 * 4 + 16 + 4 * 4 + 96 + 4 * 4 + 16
    assert C.sizeof(lib.NvLink) == 5 * 4
    assert C.sizeof(lib.RefBlock) == 20 and C.sizeof(lib.Segment) == 12
    assert C.sizeof(lib.LayoutSpec) == 8 * 4 + 8 + 8 + 8


def test_no_device_status_on_cpu(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    assert lib.load().h3c_init(0, C.byref(h)) == lib.H3C_ERR_NO_DEVICE
    n = C.c_int(-1)
    assert lib.load().h3c_device_count(C.byref(n)) == 0 and n.value == 0
    assert lib.load().h3c_last_error(None) == b"h3c: null context"
    assert lib.load().h3c_attn_fwd(None, None, None) == lib.H3C_ERR_INVALID_ARGUMENT
    assert lib.load().h3c_attn_fwd_seqshard(None, None, None) == lib.H3C_ERR_INVALID_ARGUMENT
    assert lib.load().h3c_comm_init(None, None, 2, 0) == lib.H3C_ERR_INVALID_ARGUMENT


CASES = [
    dict(seq_len=4096, frames=16, height=16, width=16, n_random=2, seed=1),
    dict(seq_len=124992, frames=31, height=48, width=84, radius_h=2, radius_w=2, n_random=4, seed=20260101),
    dict(seq_len=125632, prefix_len=640, frames=31, height=48, width=84, radius_h=2, radius_w=2, n_random=4,
         seed=20260101),
    dict(seq_len=69660, frames=43, height=30, width=54, radius_t=3, radius_h=2, radius_w=2, n_random=40, seed=7),
    dict(seq_len=800, prefix_len=100, frames=7, height=10, width=10, n_random=50, seed=5),
]


@pytest.mark.parametrize("kw", CASES)
def test_host_blockmask_equals_checker(lib, kw):
    from h3attention import BlockList, MaskSpec

    spec = MaskSpec(**{k: v for k, v in kw.items()})
    bl = BlockList.build(spec)
    rp, ci = O.blockmask_build(O.mask_spec(**kw))
    assert np.array_equal(bl.row_ptr, rp) and np.array_equal(bl.col_idx, ci)


def test_blockmask_errors(lib):
    L = lib.load()
    bad = lib.MaskSpec(seq_len=4000, block=128, frames=16, height=16, width=16, cell_t=1, cell_h=16, cell_w=32)
    nnz = C.c_int64()
    assert L.h3c_blockmask_build(C.byref(bad), None, None, 0, C.byref(nnz)) == lib.H3C_ERR_UNSUPPORTED
    neg = lib.MaskSpec(seq_len=-1, block=128)
    assert L.h3c_blockmask_build(C.byref(neg), None, None, 0, C.byref(nnz)) == lib.H3C_ERR_INVALID_ARGUMENT
    ok = lib.MaskSpec(seq_len=4096, block=128, frames=16, height=16, width=16, cell_t=1, cell_h=16, cell_w=32,
                      radius_t=1, radius_h=1, radius_w=1)
    rp = np.zeros(33, np.int32)
    ci = np.zeros(3, np.int32)
    st = L.h3c_blockmask_build(C.byref(ok), rp.ctypes.data_as(C.c_void_p), ci.ctypes.data_as(C.c_void_p), 3,
                               C.byref(nnz))
    assert st == lib.H3C_ERR_CAPACITY and nnz.value > 3


def test_workspace_size(lib):
    a = lib.AttnArgs(seq_len=1000, head_count=3, flags=lib.H3C_FUSE_PROLOGUE)
    n = C.c_size_t()
    assert lib.load().h3c_attn_workspace_size(C.byref(a), C.byref(n)) == 0
    assert n.value == 2 * 1024 * 3 * 128 * 2
    a.flags = 0
    lib.load().h3c_attn_workspace_size(C.byref(a), C.byref(n))
    assert n.value == 0


def test_density_targets():
    from h3attention.configs import CONFIGS
    from h3attention import BlockList

    d1 = BlockList.build(CONFIGS["config1"].mask_spec()).density
    d2 = BlockList.build(CONFIGS["config2"].mask_spec()).density
    assert 0.20 < d1 < 0.30
    assert 0.08 < d2 < 0.13
    assert BlockList.build(CONFIGS["config4"].mask_spec()).density == 1.0


def test_nvlink_discovery_against_a_stand_in_nvml(lib, tmp_path):
    """h3c_nvlink_query parses NVML's answers (read-only queries) into link,
    NVSwitch and version counts; checked with a stand-in NVML built from
    tests/c/fake_nvml.c, since this machine has no GPU."""
    import subprocess

    so = tmp_path / "libfake_nvml.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so), os.path.join(ROOT, "tests", "c", "fake_nvml.c")],
                   check=True)
    os.environ["H3C_NVML_LIB"] = str(so)
    try:
        L = lib.load()
        nv = lib.NvLink()
        assert L.h3c_nvlink_query(b"0000:1B:00.0", C.byref(nv)) == lib.H3C_OK
        assert (nv.available, nv.links_active, nv.links_to_switch, nv.links_to_gpu, nv.version) == (1, 18, 17, 1, 5)
        assert L.h3c_nvlink_query(b"0000:99:00.0", C.byref(nv)) == lib.H3C_ERR_NO_DEVICE
        os.environ["H3C_NVML_LIB"] = str(tmp_path / "missing.so")
        assert L.h3c_nvlink_query(b"0000:1B:00.0", C.byref(nv)) == lib.H3C_ERR_UNSUPPORTED
        assert nv.available == 0
        assert L.h3c_nvlink_query(None, C.byref(nv)) == lib.H3C_ERR_INVALID_ARGUMENT
    finally:
        del os.environ["H3C_NVML_LIB"]
