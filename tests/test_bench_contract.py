"""bench.py's checkers and its reference arm, on CPU.

* The plain PyTorch fp32 restatement that bench.py's parity leg uses
  (h3attention.torchref) agrees with the CPU oracle.
* ``bench.py --impl reference`` runs the CPU restatement without loading
  the library, on every host core, and prints the same config dict as the
  GPU arm.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _t(a):
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)


def test_torchref_prologue_matches_oracle():
    from h3attention import torchref

    S, H = 700, 3
    x = O.fill_normal_bf16((S, H, 128), 3, 1)
    w = O.fill_normal_bf16((128,), 3, 4, 1.0, 0.02)
    t, hh, ww = np.meshgrid(np.arange(7), np.arange(10), np.arange(10), indexing="ij")
    tab = O.rope_table(np.stack([t.ravel(), hh.ravel(), ww.ravel()], 1).astype(np.int32))
    for table in (tab, None):
        want = O.bf16_to_f32(O.prologue(x, w, 1e-6, table))
        got = torchref.prologue(_t(x), _t(w), 1e-6, None if table is None else _t(table)).float().numpy()
        # the sum of squares is reduced in another order: rare one-ulp flips
        # (2^-6 relative covers one ulp across a binade boundary)
        ulp = np.maximum(np.abs(want), 1e-30) * 2.0 ** -6
        assert np.all(np.abs(got - want) <= ulp + 1e-30)
        assert np.mean(got != want) < 1e-3


def test_torchref_attention_matches_oracle():
    from h3attention import BlockList, MaskSpec, torchref

    S, H = 2000, 2
    spec = MaskSpec(seq_len=S, frames=5, height=20, width=20, n_random=2, seed=4)
    bl = BlockList.build(spec)
    q, k, v = (O.fill_normal_bf16((S, H, 128), 9, st) for st in (1, 2, 3))
    want = O.attend_streaming(q, k, v, bl.row_ptr, bl.col_idx)
    qbs = torchref.sample_blocks(bl.n_blocks, 5, seed=1)
    got = torchref.attend_blocks(_t(q), _t(k), _t(v), bl.row_ptr, bl.col_idx, qbs, range(H), 128 ** -0.5)
    for (h, ib), r in got.items():
        w = want[h, ib * 128: ib * 128 + r.shape[0]]
        assert np.abs(r.numpy() - w).max() < 1e-5


def test_reference_arm_runs_the_restatement_only():
    """--impl reference: the oracle's own block list (libh3cuda.so never
    mapped), every host core although OMP_NUM_THREADS=1 (as torchrun sets it),
    and the GPU arm's config dict."""
    code = r"""
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--config", "config1", "--steps", "1", "--warmup", "3",
            "--ref-budget", "4"]
sys.path[:0] = [%r, %r]
import bench
bench.main()
maps = open("/proc/self/maps").read()
print(json.dumps({"lib_mapped": "libh3cuda" in maps}))
""" % (ROOT, os.path.join(ROOT, "minimax-h3-swift_b200"))
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(x) for x in r.stdout.strip().splitlines() if x.startswith("{")]
    line, probe = lines[0], lines[-1]
    assert probe == {"lib_mapped": False}
    assert line["impl"] == "reference" and line["extrapolated"] is True
    cores = len(os.sched_getaffinity(0))
    assert line["cpu_baseline"]["cores"] == cores
    assert line["e2e"]["h2d_bytes_per_step"] == 0

    import bench
    from h3attention import BlockList

    wl = bench._workload("config1")
    assert line["config"] == json.loads(json.dumps(bench._config(wl, BlockList.build(wl.mask_spec()), 1, "replica")))
