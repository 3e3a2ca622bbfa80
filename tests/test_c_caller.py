"""The C ABI from plain C (tests/c/render_call.c): the calls a Swift or cgo
binder makes for one render, compiled with gcc against include/h3cuda.h and
linked to libh3cuda.so.  On CPU the host half (packed layout, host block
list) must agree with the Python host mirror; on the GPU the whole render's
fused call must give the same bytes as the same call made from Python."""
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "minimax-h3-swift_b200")
BUILD = os.path.join(PKG, "_build")
EXE = os.path.join(BUILD, "render_call")
CUDA = "/usr/local/cuda"


@pytest.fixture(scope="module")
def exe():
    from h3attention import _lib

    _lib.load()  # the library must be built
    os.makedirs(BUILD, exist_ok=True)
    cc = os.environ.get("ORACLE_CC", "gcc")
    cmd = [cc, "-std=c11", "-O2", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "c", "render_call.c"), "-o", EXE, "-L", PKG,
           "-lh3cuda", "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-lm", f"-Wl,-rpath,{PKG}",
           f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return EXE


def _summary(text):
    m = re.search(r"abi (\d+) total (\d+) prefix (\d+) blocks (\d+) nnz (\d+) check (\d+)", text)
    assert m, text
    return tuple(int(x) for x in m.groups())


def _python_side():
    from h3attention import BlockList, MaskSpec
    from h3attention.layout import LatentGeometry, PackedLayout

    lay = PackedLayout(332, LatentGeometry.make(864, 480, 120), [0])
    spec = MaskSpec.for_layout(lay, radius_h=2, radius_w=2, n_random=4, seed=11)
    return lay, spec, BlockList.build(spec)


def test_host_half_matches_python(exe):
    r = subprocess.run([exe, "host"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    abi, total, prefix, nb, nnz, check = _summary(r.stdout)
    lay, spec, bl = _python_side()
    want = 0
    for c in bl.col_idx.tolist():
        want = (want * 1000003 + c) % (1 << 64)
    assert (abi, total, prefix, nb, nnz, check) == (2, lay.total_tokens, spec.prefix_len, bl.n_blocks, bl.nnz, want)
    segs = re.search(r"segments (\d+):(.*)", r.stdout)
    got = [tuple(int(x) for x in t) for t in re.findall(r"\((\d+),(\d+),(\d+)\)", segs.group(2))]
    kinds = ("text", "cond", "ref_img", "ref_audio", "audio", "video")
    assert [(a, b, kinds[k]) for a, b, k in got] == lay.segments


@pytest.mark.gpu
def test_device_render_matches_python_call(exe, gpu):
    import torch

    from h3attention import Runtime

    out_path = os.path.join(BUILD, "render_out.bin")
    r = subprocess.run([exe, "device", out_path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "device ok" in r.stdout
    lay, spec, bl = _python_side()
    S, H = lay.total_tokens, 4
    rt = Runtime.get(0)
    q, k, v = (rt.fill_normal(torch.empty((S, H, 128), dtype=torch.bfloat16, device=gpu), 41, st) for st in (1, 2, 3))
    wq, wk = (rt.fill_normal(torch.empty(128, dtype=torch.bfloat16, device=gpu), 41, st, 1.0, 0.02) for st in (4, 5))
    inv = torch.tensor([1e4 ** (-i / 16.0) for i in range(16)], dtype=torch.float32)
    table = lay.rope_table(inv, 0)
    out = torch.empty_like(q)
    rt.attn_fwd(q=q, k=k, v=v, out=out, layout="SHD", scale=128 ** -0.5, blocks=bl.on(gpu), q_norm=wq, k_norm=wk,
                eps=1e-5, rope_table=table)
    torch.cuda.synchronize()
    want = out.cpu().view(torch.int16).numpy().view(np.uint16)
    got = np.fromfile(out_path, dtype=np.uint16).reshape(S, H, 128)
    assert np.array_equal(got, want)
