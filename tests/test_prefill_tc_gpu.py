"""fr_prefill_attn on the tcgen05 kernel (FORGERT_PREFILL_KERNEL=tc, the default) and on
the mma.sync kernel (=mma): both against the fp64 oracle on the golden
fixture and across 128-row query-tile boundaries, partial tiles, GQA groups
and both head dims; then the two kernels timed on the same inputs.

Tolerance (north star): max |x - r| <= 2e-3 and
max |x - r| / max(|r|, 1e-3) <= 1e-2 on the fp16 outputs.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from oracle import oracle as O

from test_decode_gpu import assert_close, dev, nan_like

pytestmark = pytest.mark.gpu

KERNELS = ["tc", "mma"]


@pytest.fixture
def kernel(request, monkeypatch):
    monkeypatch.setenv("FORGERT_PREFILL_KERNEL", request.param)
    return request.param


def run(q, k, v, T, H, Hkv, D):
    out = nan_like(dev(q))
    A.prefill_attn_causal(dev(q), dev(k), dev(v), out, T, H, Hkv, D)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("kernel", KERNELS, indirect=True)
def test_prefill_golden(kernel):
    z = np.load(Path(__file__).parent / "golden" / "prefill_t37_h14_kv2_d64.npz")
    q, k, v = z["q"], z["k"], z["v"]
    T, H, D = q.shape
    assert_close(run(q, k, v, T, H, k.shape[1], D), z["exact"], what=f"prefill golden ({kernel})")


@pytest.mark.parametrize("kernel", KERNELS, indirect=True)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("H,Hkv", [(14, 2), (28, 4), (8, 8), (32, 2)])
@pytest.mark.parametrize("T", [1, 2, 64, 127, 128, 129, 255, 256, 700])
def test_prefill_tiles(kernel, D, H, Hkv, T):
    q, k, v = (W.normal_fp16(np.random.default_rng([T, H, Hkv, D, i, 5]), (T, n, D))
               for i, n in enumerate((H, Hkv, Hkv)))
    assert_close(run(q, k, v, T, H, Hkv, D), O.prefill_f64(q, k, v),
                 what=f"prefill {kernel} T{T} H{H} Hkv{Hkv} D{D}")


@pytest.mark.parametrize("kernel", KERNELS, indirect=True)
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_probabilities_exposed(kernel, D):
    """V rows one-hot (V[t] = e_t for t < 64): output row s is then the
    softmax row of s itself, so every probability is checked, not only their
    V-weighted sums."""
    T, H, Hkv = 64, 2, 1
    rng = np.random.default_rng(90 + D)
    q = W.normal_fp16(rng, (T, H, D))
    k = W.normal_fp16(rng, (T, Hkv, D))
    v = np.zeros((T, Hkv, D), dtype=np.float16)
    v[np.arange(T), 0, np.arange(T) + (D - 64)] = 1.0      # the last 64 dims
    assert_close(run(q, k, v, T, H, Hkv, D), O.prefill_f64(q, k, v),
                 what=f"prefill one-hot V ({kernel}, D{D})")


@pytest.mark.parametrize("kernel", KERNELS, indirect=True)
def test_prefill_long_and_large_logits(kernel):
    """T = 2048 with scaled q (logits up to ~±40): many online-softmax
    rescales and a long causal range per query tile."""
    T, H, Hkv, D = 2048, 4, 1, 128
    rng = np.random.default_rng(123)
    q = (W.normal_fp16(rng, (T, H, D)).astype(np.float32) * 3).astype(np.float16)
    k = W.normal_fp16(rng, (T, Hkv, D))
    v = W.normal_fp16(rng, (T, Hkv, D))
    assert_close(run(q, k, v, T, H, Hkv, D), O.prefill_f64(q, k, v),
                 what=f"prefill long ({kernel})")


@pytest.mark.parametrize("chunk", [0, 1, 2, 3, 7])
@pytest.mark.parametrize("T,H,Hkv,D", [(700, 14, 2, 64), (1000, 12, 2, 128), (2048, 4, 1, 128)])
def test_prefill_split_chunks(monkeypatch, chunk, T, H, Hkv, D):
    """K/V ranges of long query tiles split into units of `chunk` tiles (0 =
    unsplit; at most 4 units per query tile, so small chunks grow), merged
    by the last unit to arrive; run twice to check the counters reset."""
    monkeypatch.setenv("FORGERT_PREFILL_KERNEL", "tc")
    monkeypatch.setenv("FORGERT_PREFILL_CHUNK", str(chunk))
    q, k, v = (W.normal_fp16(np.random.default_rng([T, H, D, i, 11]), (T, n, D))
               for i, n in enumerate((H, Hkv, Hkv)))
    exact = O.prefill_f64(q, k, v)
    for rep in range(2):
        assert_close(run(q, k, v, T, H, Hkv, D), exact, what=f"split {chunk} rep {rep}")


def test_prefill_workspace_and_graph_capture(monkeypatch):
    """A split prefill inside a CUDA graph: with the workspace reserved
    first it keeps its split plan; a shape needing more than the reservation
    runs unsplit in the capture unless earlier calls grew the workspace
    further; every form is exact."""
    monkeypatch.setenv("FORGERT_PREFILL_KERNEL", "tc")
    monkeypatch.delenv("FORGERT_PREFILL_CHUNK", raising=False)
    assert A.prefill_workspace_size(8192, 28, 128) == 0            # fills the GPU unsplit
    T, H, Hkv, D = 1500, 14, 2, 64
    need = A.prefill_workspace_size(T, H, D)
    assert need > 0
    A.reserve_workspace(need)
    q, k, v = (W.normal_fp16(np.random.default_rng([T, i, 12]), (T, n, D))
               for i, n in enumerate((H, Hkv, Hkv)))
    exact = O.prefill_f64(q, k, v)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = nan_like(qd)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        A.prefill_attn_causal(qd, kd, vd, out, T, H, Hkv, D, s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        A.prefill_attn_causal(qd, kd, vd, out, T, H, Hkv, D, torch.cuda.current_stream())
    for _ in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert_close(out.cpu().numpy(), exact, what="captured split prefill")
    # a shape whose split plan needs more workspace than exists: unsplit in capture
    T2, H2, Hkv2, D2 = 2048, 12, 2, 128
    q2, k2, v2 = (W.normal_fp16(np.random.default_rng([T2, i, 13]), (T2, n, D2))
                  for i, n in enumerate((H2, Hkv2, Hkv2)))
    assert A.prefill_workspace_size(T2, H2, D2) > need
    out2 = nan_like(dev(q2))
    q2d, k2d, v2d = dev(q2), dev(k2), dev(v2)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=s):
        A.prefill_attn_causal(q2d, k2d, v2d, out2, T2, H2, Hkv2, D2, torch.cuda.current_stream())
    g2.replay()
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert_close(out2.cpu().numpy(), O.prefill_f64(q2, k2, v2), what="capture fallback")
    del g, g2


def test_prefill_kernels_timed(monkeypatch):
    """Both kernels on T = 2048 and 8192, H28 Hkv4 D128 (CUDA events, 10
    launches after 3 warm-ups).  Useful causal flops = 2 * 2 * H * D * T(T+1)/2."""
    H, Hkv, D = 28, 4, 128
    res = {}
    for T in (2048, 8192):
        rng = np.random.default_rng(T)
        q = torch.from_numpy(W.normal_fp16(rng, (T, H, D))).cuda()
        k = torch.from_numpy(W.normal_fp16(rng, (T, Hkv, D))).cuda()
        v = torch.from_numpy(W.normal_fp16(rng, (T, Hkv, D))).cuda()
        outs = {}
        for name in KERNELS:
            monkeypatch.setenv("FORGERT_PREFILL_KERNEL", name)
            out = torch.empty_like(q)
            for _ in range(3):
                A.prefill_attn_causal(q, k, v, out, T, H, Hkv, D)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                A.prefill_attn_causal(q, k, v, out, T, H, Hkv, D)
            e1.record()
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / 10
            flops = 2.0 * 2 * H * D * T * (T + 1) / 2
            res[f"{name}_T{T}"] = {"us": round(us, 1), "tflops": round(flops / us / 1e6, 1)}
            outs[name] = out.float().cpu().numpy()
        assert A.device_error() == 0
        for name in KERNELS[1:]:
            a, r = O.max_errors(outs[KERNELS[0]], outs[name], 1e-3)
            assert a <= 2e-3, (T, name, a, r)
    print("\n" + json.dumps({"prefill_kernels": res}))


@pytest.mark.parametrize("kernel", KERNELS, indirect=True)
@pytest.mark.parametrize("T,H,Hkv,D", [(300, 8, 2, 128), (2048, 4, 1, 64)])
def test_prefill_output_4_byte_aligned(kernel, T, H, Hkv, D):
    """out 4-byte but not 16-byte aligned (the C ABI's minimum): the kernels
    store with 4-byte writes, unsplit and through the split merge."""
    q, k, v = (W.normal_fp16(np.random.default_rng([T, D, i, 14]), (T, n, D))
               for i, n in enumerate((H, Hkv, Hkv)))
    buf = torch.full((T * H * D + 8,), float("nan"), dtype=torch.float16, device="cuda")
    out = buf[2:2 + T * H * D].view(T, H, D)           # base + 4 bytes
    assert out.data_ptr() % 16 == 4
    A.prefill_attn_causal(dev(q), dev(k), dev(v), out, T, H, Hkv, D)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert_close(out.cpu().numpy(), O.prefill_f64(q, k, v), what=f"prefill 4B-aligned out ({kernel})")
    assert torch.isnan(buf[:2]).all() and torch.isnan(buf[2 + T * H * D:]).all()
