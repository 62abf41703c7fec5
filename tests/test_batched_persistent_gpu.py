"""GPU parity of the persistent batched decode kernel (fr_decode_attn_batched).

The batched entry point spreads all units' 64-row K/V tiles evenly over a
persistent grid (stream-K): a unit can be shared by many CTAs, whose pieces
are merged by the last one to finish.  Checked against the fp64 oracle at the
engine tolerance (max abs 2e-3, max rel 1e-2 with a 1e-3 floor):

* GQA groups of 1, 7, 8, 16 and 20 query heads (one and two 8-head tiles,
  several head groups per kv head), head_dim 64 and 128;
* ragged lengths with 0, 1, 63, 64, 65 rows, pools whose rows between
  sequences hold NaN;
* one long sequence (one unit spread over dozens of CTAs), fewer tiles than
  CTAs, the largest batch the kernel takes (512) and one more (the split
  kernel's grid takes over);
* repeated calls and CUDA-graph replays with new inputs (the per-unit merge
  counters re-arm between calls), with and without launch overlap;
* the split-kernel grid selected by FORGERT_BATCHED_KERNEL=split (a fresh
  process) on the same inputs.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from forgert_b200 import _lib
from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
ATOL, RTOL, EPS = 2e-3, 1e-2, 1e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_close(x, ref, what=""):
    a, r = O.max_errors(x, ref, EPS)
    assert np.isfinite(np.asarray(x, np.float64)).all(), f"{what}: non-finite output"
    assert a <= ATOL and r <= RTOL, f"{what}: max abs {a:.3g}, max rel {r:.3g}"


def make_batch(seed, H, Hkv, D, lens, gap_rows=0):
    rng = np.random.default_rng(seed)
    B = len(lens)
    q = W.normal_fp16(rng, (B, H, D))
    ks = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
    vs = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
    offsets, pk, pv, row = [], [], [], 0
    gap = np.full((gap_rows, Hkv, D), np.nan, np.float16)
    for k, v in zip(ks, vs):
        offsets.append(row)
        pk += [k, gap]
        pv += [v, gap]
        row += k.shape[0] + gap_rows
    pool_k = np.concatenate(pk) if row else np.zeros((1, Hkv, D), np.float16)
    pool_v = np.concatenate(pv) if row else np.zeros((1, Hkv, D), np.float16)
    return q, ks, vs, pool_k, pool_v, np.asarray(offsets, np.int64), max(row, 1)


def run(q, pool_k, pool_v, offsets, lens, rows, stream=None):
    B, H, D = q.shape
    Hkv = pool_k.shape[1]
    qd, kd, vd = dev(q), dev(pool_k), dev(pool_v)
    offs, lens_d = dev(offsets), dev(np.asarray(lens, np.int32))
    out = torch.full_like(qd, float("nan"))
    A.decode_attn_batched(qd, kd, vd, offs, lens_d, out, B, H, Hkv, D, rows,
                          int(max(lens)), stream)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("H,Hkv,D", [(28, 4, 128), (14, 2, 64), (8, 8, 128), (16, 2, 128),
                                     (16, 1, 64), (32, 2, 128), (40, 2, 64)])
def test_ragged_shapes(H, Hkv, D):
    lens = [1, 64, 65, 300, 0, 2049, 17, 63, 1500, 4096, 129]
    q, ks, vs, pk, pv, offs, rows = make_batch(11, H, Hkv, D, lens, gap_rows=37)
    out = run(q, pk, pv, offs, lens, rows)
    assert_close(out, O.batched_f64(q, ks, vs, lens), what=f"H{H} Hkv{Hkv} D{D}")
    assert np.all(out[4] == 0), "kv_len 0 yields zeros"


def test_one_long_sequence_many_pieces():
    """One sequence of 131072 rows (4 kv heads): each unit is cut into pieces
    over dozens of CTAs and merged by the last one."""
    lens = [131072]
    q, ks, vs, pk, pv, offs, rows = make_batch(12, 28, 4, 128, lens)
    out = run(q, pk, pv, offs, lens, rows)
    assert_close(out, O.batched_f64(q, ks, vs, lens), what="one long sequence")


def test_fewer_tiles_than_ctas():
    lens = [1, 0, 2]
    q, ks, vs, pk, pv, offs, rows = make_batch(13, 14, 2, 64, lens, gap_rows=5)
    out = run(q, pk, pv, offs, lens, rows)
    assert_close(out, O.batched_f64(q, ks, vs, lens), what="tiny batch")


@pytest.mark.parametrize("B", [512, 513])
def test_largest_batch_and_one_more(B):
    rng = np.random.default_rng(14)
    lens = rng.integers(0, 300, size=B)
    q, ks, vs, pk, pv, offs, rows = make_batch(15, 8, 1, 128, lens, gap_rows=3)
    out = run(q, pk, pv, offs, lens, rows)
    assert_close(out, O.batched_f64(q, ks, vs, lens), what=f"B={B}")


@pytest.mark.parametrize("overlap", [0, 1])
def test_repeated_and_graph_replayed(overlap):
    """Three eager calls and three replays of a captured call, each with new q
    (and new K/V values in place): the merge counters re-arm every call."""
    lib = _lib.load()
    prev = lib.fr_set_launch_overlap(overlap)
    try:
        H, Hkv, D = 28, 4, 128
        rng = np.random.default_rng(16)
        lens = rng.integers(1024, 8193, size=16)
        q, ks, vs, pk, pv, offs, rows = make_batch(17, H, Hkv, D, lens)
        B = len(lens)
        kd, vd, offs_d = dev(pk), dev(pv), dev(offs)
        lens_d = dev(np.asarray(lens, np.int32))
        qd = dev(q)
        out = torch.empty_like(qd)
        stream = torch.cuda.Stream()
        A.reserve_workspace(A.decode_workspace_size(B, H, Hkv, D, int(max(lens))))

        def call(s):
            A.decode_attn_batched(qd, kd, vd, offs_d, lens_d, out, B, H, Hkv, D, rows,
                                  int(max(lens)), s)

        def check(what):
            torch.cuda.synchronize()
            assert A.device_error() == 0
            kk = kd.cpu().numpy()
            vv = vd.cpu().numpy()
            ks_ = [kk[o:o + n] for o, n in zip(offs, lens)]
            vs_ = [vv[o:o + n] for o, n in zip(offs, lens)]
            assert_close(out.cpu().numpy(), O.batched_f64(qd.cpu().numpy(), ks_, vs_, lens),
                         what=what)

        with torch.cuda.stream(stream):
            for i in range(3):
                qd.copy_(dev(W.normal_fp16(rng, q.shape)))
                call(stream)
                check(f"eager call {i}")
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                call(torch.cuda.current_stream())
            for i in range(3):
                qd.copy_(dev(W.normal_fp16(rng, q.shape)))
                kd.mul_(-1.0)
                g.replay()
                check(f"replay {i}")
    finally:
        lib.fr_set_launch_overlap(prev)


_SPLIT_PROCESS = r"""
import json, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from forgert_b200 import attention as A
from forgert_b200 import workloads as W
lens = [1, 64, 65, 300, 0, 2049, 17, 1500]
rng = np.random.default_rng(5)
H, Hkv, D = 28, 4, 128
B = len(lens)
q = W.normal_fp16(rng, (B, H, D))
ks = [W.normal_fp16(rng, (n, Hkv, D)) for n in lens]
vs = [W.normal_fp16(rng, (n, Hkv, D)) for n in lens]
offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
out = torch.full((B, H, D), float("nan"), dtype=torch.float16, device="cuda")
A.decode_attn_batched(d(q), d(np.concatenate(ks)), d(np.concatenate(vs)), d(offs),
                      d(np.asarray(lens, np.int32)), out, B, H, Hkv, D, int(sum(lens)), max(lens))
torch.cuda.synchronize()
np.save(sys.argv[2], out.cpu().numpy())
print(json.dumps({"err": A.device_error()}))
"""


def test_split_grid_selected_by_environment(tmp_path):
    """FORGERT_BATCHED_KERNEL=split keeps the split kernel's grid for batched
    calls (read once per process); its output matches the oracle too."""
    import os
    env = dict(os.environ, FORGERT_BATCHED_KERNEL="split")
    f = tmp_path / "out.npy"
    r = subprocess.run([sys.executable, "-c", _SPLIT_PROCESS, str(ROOT), str(f)], env=env,
                       capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-3000:]
    assert json.loads(r.stdout.strip().splitlines()[-1])["err"] == 0
    lens = [1, 64, 65, 300, 0, 2049, 17, 1500]
    rng = np.random.default_rng(5)
    q = W.normal_fp16(rng, (8, 28, 128))
    ks = [W.normal_fp16(rng, (n, 4, 128)) for n in lens]
    vs = [W.normal_fp16(rng, (n, 4, 128)) for n in lens]
    assert_close(np.load(f), O.batched_f64(q, ks, vs, lens), what="split grid")


def test_bitwise_repeatable():
    """The contributor that completes a unit's count merges it, and which one
    that is varies from call to call; the merge reads the pieces in a fixed
    order, so repeated calls give identical bits."""
    rng = np.random.default_rng(18)
    lens = rng.integers(1024, 8193, size=32)
    q, ks, vs, pk, pv, offs, rows = make_batch(19, 28, 4, 128, lens)
    first = run(q, pk, pv, offs, lens, rows)
    for _ in range(4):
        assert np.array_equal(run(q, pk, pv, offs, lens, rows), first)
    assert_close(first, O.batched_f64(q, ks, vs, lens), what="repeatable batch")
