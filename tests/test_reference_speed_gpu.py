"""The reference's own GPU code and this library, timed side by side on one B200.

The reference's kernels are compiled for sm_100a from its sources
(oracle/Makefile -> oracle/_ref, -O3 --use_fast_math as its CMakeLists.txt)
and run on the same device buffers as ours:

* decode attention: decode_attn_v4_flash (kernels/attention_decode.cu:418-556)
  against fr_decode_attn on the cfg2 shape (H12 Hkv2 D128) at kv_len 512,
  2048, 4096 and 16384, 28 layer caches per kv_len, each group of 28 calls
  captured as one CUDA graph on one stream, L2 flushed (256 MiB write)
  before each replay, CUDA events around the replay;
* decode prologue: the six launches of runtime/executor.cpp:135-152 (three
  bias_add_broadcast, rope_v2_fused, two device copies) against one
  fr_qkv_bias_rope_append, for one decode token of Qwen2-0.5B (H14 Hkv2 D64)
  and of the cfg2 shape, 100 tokens per CUDA graph.

Each test prints one JSON line with the timings (read with pytest -s) and
asserts only a wide margin, so that a slow box does not fail it.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

L2_FLUSH_BYTES = 256 << 20


@pytest.fixture(scope="module")
def ref():
    lib = O.load_ref()
    if lib is None:
        pytest.skip("oracle/_ref not built")
    return lib


def _graph(fn, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def _time_groups(groups, reps, flush, stream):
    """ms per group (summed over reps): each group is one CUDA graph (so host
    overhead is not timed), replayed after a flush."""
    graphs = {k: _graph(fn, stream) for k, fn in groups.items()}
    ms = {k: 0.0 for k in groups}
    with torch.cuda.stream(stream):
        for _ in range(reps):
            for i, (k, g) in enumerate(graphs.items()):
                flush.fill_(i & 0xFF)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
                e1.synchronize()
                ms[k] += e0.elapsed_time(e1)
    return ms


def test_decode_attention_vs_reference_v4(ref):
    L, S, H, Hkv, D = 28, W.CFG2_MAX_SEQ, 12, 2, 128
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    cache = torch.empty((L, 2, S, Hkv, D), dtype=torch.float16, device=dev).normal_(generator=g)
    q = torch.empty((L, H, D), dtype=torch.float16, device=dev).normal_(generator=g)
    out_ref = torch.empty_like(q)
    out = torch.empty_like(q)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream

    def ref_group(kv):
        def fn():
            for l in range(L):
                ref.ref_decode_attn_v4_flash(q[l].data_ptr(), cache[l, 0].data_ptr(),
                                             cache[l, 1].data_ptr(), out_ref[l].data_ptr(),
                                             H, Hkv, D, kv, sp)
        return fn

    def our_group(kv):
        def fn():
            for l in range(L):
                A.decode_attn_v4_flash(q[l], cache[l, 0], cache[l, 1], out[l], H, Hkv, D, kv,
                                       stream)
        return fn

    kvs = W.CFG2_KV_LENS
    for fn in [ref_group(k) for k in kvs] + [our_group(k) for k in kvs]:
        with torch.cuda.stream(stream):
            fn()
    torch.cuda.synchronize()
    reps = 5
    t_ref = _time_groups({k: ref_group(k) for k in kvs}, reps, flush, stream)
    t_our = _time_groups({k: our_group(k) for k in kvs}, reps, flush, stream)
    assert A.device_error() == 0
    res = {}
    for k in kvs:
        us_r = t_ref[k] * 1e3 / (reps * L)
        us_o = t_our[k] * 1e3 / (reps * L)
        gb = W.decode_bytes([k], H, Hkv, D) / 1e9
        res[k] = {"ref_v4_us": round(us_r, 2), "ours_us": round(us_o, 2),
                  "ref_v4_gbs": round(gb / (us_r * 1e-6), 1), "ours_gbs": round(gb / (us_o * 1e-6), 1),
                  "speedup": round(us_r / us_o, 1)}
    print("\n" + json.dumps({"decode_attention_graph_cfg2": res}))
    # the same outputs, within the parity tolerance
    a, r = O.max_errors(out.float().cpu().numpy(), out_ref.float().cpu().numpy(), 1e-3)
    assert a <= 2e-3 and r <= 1e-2, (a, r)
    for k in kvs:
        assert res[k]["speedup"] > 5, res[k]


@pytest.mark.parametrize("tables", ["exact", "device"])
@pytest.mark.parametrize("H,Hkv,D", [(14, 2, 64), (12, 2, 128)])
def test_prologue_vs_reference_sequence(ref, H, Hkv, D, tables):
    """The fused prologue leaves q, k, v and both cache rows bit-identical to
    the reference's six launches, with either table set (both paths read the
    same tables); then both are timed."""
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(77)
    S, pos, T = 16384, 16000, 1
    q0 = torch.from_numpy(W.normal_fp16(rng, (T, H, D))).to(dev)
    k0 = torch.from_numpy(W.normal_fp16(rng, (T, Hkv, D))).to(dev)
    v0 = torch.from_numpy(W.normal_fp16(rng, (T, Hkv, D))).to(dev)
    bq = torch.from_numpy(W.normal_fp16(rng, (H * D,))).to(dev)
    bk = torch.from_numpy(W.normal_fp16(rng, (Hkv * D,))).to(dev)
    bv = torch.from_numpy(W.normal_fp16(rng, (Hkv * D,))).to(dev)
    make = A.rope_precompute_tables if tables == "exact" else A.rope_tables_device
    cos_t, sin_t = make(S, D, W.ROPE_THETA, device=dev)
    kc_r = torch.zeros((S, Hkv, D), dtype=torch.float16, device=dev)
    vc_r = torch.zeros_like(kc_r)
    kc_o, vc_o = torch.zeros_like(kc_r), torch.zeros_like(kc_r)
    bufs_r = [t.clone() for t in (q0, k0, v0)]
    bufs_o = [t.clone() for t in (q0, k0, v0)]
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream
    row = Hkv * D

    def ref_seq():
        qr, kr, vr = bufs_r
        ref.ref_bias_add_broadcast(qr.data_ptr(), bq.data_ptr(), T, H * D, sp)
        ref.ref_bias_add_broadcast(kr.data_ptr(), bk.data_ptr(), T, row, sp)
        ref.ref_bias_add_broadcast(vr.data_ptr(), bv.data_ptr(), T, row, sp)
        ref.ref_rope_v2_fused(qr.data_ptr(), kr.data_ptr(), cos_t.data_ptr(), sin_t.data_ptr(), T,
                              H, Hkv, D, pos, sp)
        kc_r[pos:pos + T].copy_(kr.view(T, Hkv, D), non_blocking=True)
        vc_r[pos:pos + T].copy_(vr.view(T, Hkv, D), non_blocking=True)

    def our_seq():
        qo, ko, vo = bufs_o
        A.qkv_bias_rope_append(qo, ko, vo, bq, bk, bv, kc_o, vc_o, cos_t, sin_t, T, H, Hkv, D,
                               pos, stream)

    # parity, one application from the same inputs
    with torch.cuda.stream(stream):
        ref_seq()
        our_seq()
    torch.cuda.synchronize()
    assert A.device_error() == 0
    pairs = [(bufs_o[0], bufs_r[0]), (bufs_o[1], bufs_r[1]), (bufs_o[2], bufs_r[2]),
             (kc_o, kc_r), (vc_o, vc_r)]
    exact = 0
    total = 0
    for got, want in pairs:
        exact += int((got.view(torch.int16) == want.view(torch.int16)).sum())
        total += got.numel()
    assert exact == total, f"{total - exact} of {total} fp16 values differ from the reference's"
    for got, want in pairs:
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))

    # timing: 100 tokens' prologues back to back in one CUDA graph (device
    # time, no host overhead; in-place updates keep going), replayed 20 times
    per_graph, reps = 100, 20

    def timed(fn):
        def body():
            for _ in range(per_graph):
                fn()
        g = _graph(body, stream)
        with torch.cuda.stream(stream):
            g.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * per_graph)

    us_ref = timed(ref_seq)
    us_our = timed(our_seq)
    assert A.device_error() == 0
    print("\n" + json.dumps({"prologue_per_layer_token": {
        "shape": f"H{H} Hkv{Hkv} D{D}", "tables": tables, "ref_6_launches_us": round(us_ref, 2),
        "fused_us": round(us_our, 2), "speedup": round(us_ref / us_our, 1),
        "bit_exact_fraction": round(exact / total, 6)}}))
    assert us_our < us_ref


@pytest.mark.parametrize("H,Hkv,D,T", [(14, 2, 64, 512), (14, 2, 64, 2048), (28, 4, 128, 2048)])
def test_prefill_vs_reference(ref, H, Hkv, D, T):
    """Causal prefill over T positions: the reference's prefill_attn_causal
    (kernels/attention_decode.cu:563-619, one thread per (head, position))
    against fr_prefill_attn (the split kernel, one 'sequence' per query
    position), each as a CUDA graph on the same buffers, 20 replays."""
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(T + D)
    q = torch.from_numpy(W.normal_fp16(rng, (T, H, D))).to(dev)
    k = torch.from_numpy(W.normal_fp16(rng, (T, Hkv, D))).to(dev)
    v = torch.from_numpy(W.normal_fp16(rng, (T, Hkv, D))).to(dev)
    out_ref = torch.empty_like(q)
    out = torch.empty_like(q)
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream

    def ref_call():
        ref.ref_prefill_attn_causal(q.data_ptr(), k.data_ptr(), v.data_ptr(), out_ref.data_ptr(),
                                    T, H, Hkv, D, sp)

    def our_call():
        A.prefill_attn_causal(q, k, v, out, T, H, Hkv, D, stream)

    res = {}
    for name, fn in (("ref", ref_call), ("ours", our_call)):
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        g = _graph(fn, stream)
        with torch.cuda.stream(stream):
            g.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(20):
                g.replay()
            e1.record(stream)
        e1.synchronize()
        res[name] = e0.elapsed_time(e1) * 1e3 / 20
    assert A.device_error() == 0
    a, r = O.max_errors(out.float().cpu().numpy(), out_ref.float().cpu().numpy(), 1e-3)
    assert a <= 2e-3 and r <= 1e-2, (a, r)
    print("\n" + json.dumps({"prefill": {"shape": f"T{T} H{H} Hkv{Hkv} D{D}",
                                         "ref_us": round(res["ref"], 1),
                                         "ours_us": round(res["ours"], 1),
                                         "speedup": round(res["ref"] / res["ours"], 1)}}))
    assert res["ours"] < res["ref"]
