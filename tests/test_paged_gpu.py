"""GPU parity tests of the paged-KV decode (fr_decode_attn_paged), through the C ABI.

Each case lays seeded per-sequence caches out as pages handed out in a
shuffled order (forgert_b200.workloads.paginate), fills every row that no
sequence owns with NaN, and compares the fp16 output with

* the CPU oracle (oracle.paged_f64: rows gathered back into one cache per
  sequence, fp64) at max |x - r| <= 2e-3 and max |x - r| / max(|r|, 1e-3) <= 1e-2;
* the contiguous-pool batched call on the same sequences, at the same
  tolerance (the pooled layout runs the persistent batched kernel, which
  splits the rows differently).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from forgert_b200._lib import ForgeRTError
from oracle import oracle as O

from test_decode_gpu import assert_close, dev, nan_like, run_batched

pytestmark = pytest.mark.gpu


def run_paged(q, k_pages, v_pages, table, lens, page_size, max_kv_len=None, width=None):
    B, H, D = q.shape
    Hkv = k_pages.shape[2]
    qd = dev(q)
    out = nan_like(qd)
    tbl = dev(np.ascontiguousarray(table, np.int32))
    lens_d = dev(np.asarray(lens, np.int32))
    mk = int(max(lens)) if max_kv_len is None else max_kv_len
    A.decode_attn_paged(qd, dev(k_pages), dev(v_pages), tbl, lens_d, out, B, H, Hkv, D,
                        page_size, k_pages.shape[0], table.shape[1] if width is None else width,
                        mk)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return out.cpu().numpy()


def ragged(rng, lens, H, Hkv, D):
    q = W.normal_fp16(rng, (len(lens), H, D))
    ks = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
    vs = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
    return q, ks, vs


@pytest.mark.parametrize("page_size", [16, 32, 48, 64, 128, 256])
@pytest.mark.parametrize("D,H,Hkv", [(128, 28, 4), (64, 14, 2)])
def test_paged_matches_oracle_and_pool(page_size, D, H, Hkv):
    rng = np.random.default_rng(100 + page_size + D)
    lens = np.array([1, page_size - 1, page_size, page_size + 1, 0, 2049, 17, 700, 3 * page_size],
                    np.int32)
    q, ks, vs = ragged(rng, lens, H, Hkv, D)
    kp, vp, table = W.paginate(ks, vs, page_size, seed=page_size, spare_pages=5)
    # Entries past each sequence's pages are never read: make them hostile.
    table = table.copy()
    table[table < 0] = np.int32(2**30)
    out = run_paged(q, kp, vp, table, lens, page_size)
    ref = O.paged_f64(q, kp, vp, table, lens, page_size)
    assert_close(out, ref, what=f"paged page_size={page_size} D={D}")
    assert np.all(out[4] == 0), "kv_len 0 yields zeros"
    # The pooled layout runs the persistent batched kernel (a different split
    # of the same rows), so the two agree to the tolerance, not bit for bit.
    pooled = run_batched(q, ks, vs, lens, gap_rows=3)
    assert_close(out, pooled, what=f"paged vs pooled page_size={page_size} D={D}")


def test_paged_out_of_pool_ids_read_as_zero_rows():
    """A page id outside [0, num_pages) inside a sequence's range reads zeros
    (no fault): the result equals the oracle over a cache with those rows zero."""
    rng = np.random.default_rng(9)
    H, Hkv, D, P = 12, 2, 128, 32
    lens = np.array([200, 96], np.int32)
    q, ks, vs = ragged(rng, lens, H, Hkv, D)
    kp, vp, table = W.paginate(ks, vs, P, seed=3)
    table = table.copy()
    table[0, 2] = kp.shape[0] + 7       # rows 64..95 of sequence 0
    table[1, 1] = -3                    # rows 32..63 of sequence 1
    out = run_paged(q, kp, vp, table, lens, P)
    ks[0][64:96] = 0
    vs[0][64:96] = 0
    ks[1][32:64] = 0
    vs[1][32:64] = 0
    assert_close(out, O.batched_f64(q, ks, vs, lens), what="out-of-pool page ids")


def test_paged_single_long_sequence_uses_cluster_merge():
    """One 40000-position sequence: many splits, fused cluster merge, 16-row pages."""
    rng = np.random.default_rng(11)
    H, Hkv, D, P = 28, 4, 128, 16
    lens = np.array([40000], np.int32)
    q, ks, vs = ragged(rng, lens, H, Hkv, D)
    kp, vp, table = W.paginate(ks, vs, P, seed=5, spare_pages=11)
    out = run_paged(q, kp, vp, table, lens, P)
    assert_close(out, O.paged_f64(q, kp, vp, table, lens, P), what="paged long")


@pytest.mark.parametrize("page_size", [16, 64])
def test_cfg3_paged_full(page_size):
    lens, q, ks, vs = W.cfg3_inputs()
    kp, vp, table = W.paginate(ks, vs, page_size, seed=1)
    out = run_paged(q, kp, vp, table, lens, page_size)
    assert_close(out, O.paged_f64(q, kp, vp, table, lens, page_size), what="cfg3 paged")


def test_paged_graph_capture_replays():
    rng = np.random.default_rng(12)
    H, Hkv, D, P = 28, 4, 128, 32
    lens = np.array([3000, 17, 1200, 64], np.int32)
    q, ks, vs = ragged(rng, lens, H, Hkv, D)
    kp, vp, table = W.paginate(ks, vs, P, seed=2)
    qd, kd, vd = dev(q), dev(kp), dev(vp)
    tbl, lens_d = dev(table), dev(lens)
    out = nan_like(qd)
    args = (qd, kd, vd, tbl, lens_d, out, len(lens), H, Hkv, D, P, kp.shape[0], table.shape[1],
            int(lens.max()))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        A.decode_attn_paged(*args, stream=s)          # plans + sizes the workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        A.decode_attn_paged(*args, stream=s)
    out.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert_close(out.cpu().numpy(), O.paged_f64(q, kp, vp, table, lens, P), what="paged graph")


def test_paged_invalid_arguments():
    q = torch.zeros((1, 8, 64), dtype=torch.float16, device="cuda")
    kp = torch.zeros((4, 16, 2, 64), dtype=torch.float16, device="cuda")
    tbl = torch.zeros((1, 4), dtype=torch.int32, device="cuda")
    lens = torch.ones((1,), dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    ok = (q, kp, kp, tbl, lens, out, 1, 8, 2, 64, 16, 4, 4, 64)
    A.decode_attn_paged(*ok)
    torch.cuda.synchronize()
    for bad, what in [
        (dict(page_size=8), "page size not a multiple of 16"),
        (dict(max_kv_len=65), "max_kv_len beyond the table"),
        (dict(num_pages=0), "empty pool"),
        (dict(D=96), "head_dim"),
    ]:
        a = list(ok)
        if "page_size" in bad:
            a[10] = bad["page_size"]
        if "max_kv_len" in bad:
            a[13] = bad["max_kv_len"]
        if "num_pages" in bad:
            a[11] = bad["num_pages"]
        if "D" in bad:
            a[9] = bad["D"]
        with pytest.raises(ForgeRTError):
            A.decode_attn_paged(*a)
