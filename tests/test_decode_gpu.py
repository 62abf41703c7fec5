"""GPU parity tests of the decode-attention path, through the C ABI.

Every case runs libforgert_b200.so on seeded inputs and compares the fp16
output with the CPU oracle (oracle/oracle.py, fp64) at

    max |x - r| <= 2e-3   and   max |x - r| / max(|r|, 1e-3) <= 1e-2

(the tolerance of the engine's specification).  Where the reference's own GPU
kernel was built (oracle/_ref), it runs on the same inputs too.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from forgert_b200._lib import ForgeRTError
from oracle import oracle as O

ATOL = 2e-3
RTOL = 1e-2
EPS = 1e-3

pytestmark = pytest.mark.gpu

GOLDEN_DECODE = [
    "ref_h8_kv2_d64_len128", "ref_h8_kv2_d64_len1", "ref_h8_kv2_d128_len128",
    "gqa7_d128_len33", "gqa16_d64_len200", "mha_d128_len100", "gqa6_d128_len300",
]


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def nan_like(t: torch.Tensor) -> torch.Tensor:
    return torch.full_like(t, float("nan"))


def assert_close(x, ref, atol=ATOL, rtol=RTOL, what=""):
    a, r = O.max_errors(x, ref, EPS)
    assert np.isfinite(np.asarray(x, np.float64)).all(), f"{what}: non-finite output"
    assert a <= atol and r <= rtol, f"{what}: max abs {a:.3g}, max rel {r:.3g}"


def decode(q, k, v, kv_len=None):
    H, D = q.shape
    Hkv = k.shape[1]
    T = k.shape[0] if kv_len is None else kv_len
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = nan_like(qd)
    A.decode_attn_v4_flash(qd, kd, vd, out, H, Hkv, D, T)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("name", GOLDEN_DECODE)
def test_golden_fixtures(name):
    from pathlib import Path
    z = np.load(Path(__file__).parent / "golden" / f"{name}.npz")
    out = decode(z["q"], z["k"], z["v"])
    assert_close(out, z["exact"], what=f"{name} vs exact")
    assert_close(out, z["ref_f32"], what=f"{name} vs reference cpu_decode_attn")


def test_cfg1_full():
    q, k, v = W.cfg1_inputs()
    assert_close(decode(q, k, v), O.decode_f64(q, k, v), what="cfg1")


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("H,Hkv", [(4, 4), (8, 2), (14, 2), (16, 2), (28, 4), (32, 2), (40, 2)])
@pytest.mark.parametrize("kv_len", [1, 2, 15, 16, 17, 63, 64, 65, 129, 1000, 4097])
def test_shapes_and_lengths(D, H, Hkv, kv_len):
    seed = [D, H, Hkv, kv_len]
    q, k, v = W.decode_inputs(seed, H, Hkv, D, kv_len)
    assert_close(decode(q, k, v), O.decode_f64(q, k, v), what=f"D{D} H{H} Hkv{Hkv} T{kv_len}")


def test_prefix_of_longer_cache():
    """kv_len shorter than the cache view: rows past kv_len must be ignored."""
    q, k, v = W.decode_inputs(7, 12, 2, 128, 700)
    k[500:] = np.float16(60000)   # huge values past kv_len would dominate if read
    assert_close(decode(q, k, v, kv_len=500), O.decode_f64(q, k[:500], v[:500]), what="prefix")


@pytest.mark.parametrize("layer", [0, 27])
@pytest.mark.parametrize("kv_len", W.CFG2_KV_LENS)
def test_cfg2_layers_full_size(layer, kv_len):
    k, v = W.cfg2_layer_kv(layer)
    q = W.cfg2_layer_q(layer)
    assert_close(decode(q, k, v, kv_len), O.decode_f64(q, k, v, kv_len), what=f"cfg2 L{layer} T{kv_len}")


def test_properties_constant_v_and_zero_q():
    """Softmax weights sum to one: constant V rows give that constant back;
    q = 0 gives the mean of V."""
    q, k, v = W.decode_inputs(9, 14, 2, 64, 3000)
    vc = np.broadcast_to(v[:1], v.shape).copy()
    out = decode(q, k, vc)
    G = 7
    for h in range(14):
        assert np.allclose(out[h], v[0, h // G].astype(np.float64), atol=1e-3)
    out0 = decode(np.zeros_like(q), k, v)
    mean = v.astype(np.float64).mean(axis=0)   # [Hkv, D]
    assert_close(out0, np.repeat(mean, G, axis=0), what="q=0 mean")


def test_batched_ragged_small():
    rng = np.random.default_rng(5)
    H, Hkv, D = 28, 4, 128
    lens = np.array([1, 64, 65, 300, 0, 2049, 17, 1500], np.int32)
    B = len(lens)
    q = W.normal_fp16(rng, (B, H, D))
    ks = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
    vs = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
    out = run_batched(q, ks, vs, lens, gap_rows=37)
    ref = O.batched_f64(q, ks, vs, lens)
    assert_close(out, ref, what="batched ragged")
    assert np.all(out[4] == 0), "kv_len 0 yields zeros"


def run_batched(q, ks, vs, lens, gap_rows=0):
    """Packs the sequences into one KV pool, separated by `gap_rows` rows of
    NaN (rows past a sequence's end must never reach the output)."""
    B, H, D = q.shape
    Hkv = ks[0].shape[1] if ks else 1
    offsets, parts_k, parts_v, row = [], [], [], 0
    nan_rows = np.full((gap_rows, Hkv, D), np.nan, np.float16)
    for k, v in zip(ks, vs):
        offsets.append(row)
        parts_k += [k, nan_rows]
        parts_v += [v, nan_rows]
        row += k.shape[0] + gap_rows
    kd, vd = dev(np.concatenate(parts_k)), dev(np.concatenate(parts_v))
    offs = dev(np.asarray(offsets, np.int64))
    lens_d = dev(np.asarray(lens, np.int32))
    qd = dev(q)
    out = nan_like(qd)
    A.decode_attn_batched(qd, kd, vd, offs, lens_d, out, B, H, Hkv, D, row, int(max(lens)))
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return out.cpu().numpy()


def test_cfg3_batched_full():
    lens, q, ks, vs = W.cfg3_inputs()
    out = run_batched(q, ks, vs, lens)
    assert_close(out, O.batched_f64(q, ks, vs, lens), what="cfg3")


def test_cfg4_long_context_and_partial_merge():
    q, k, v = W.cfg4_inputs()
    H, D = q.shape
    Hkv = k.shape[1]
    exact = O.decode_f64(q, k, v)
    assert_close(decode(q, k, v), exact, what="cfg4 single call")
    # KV range split in 8 (what 8 GPUs each hold), one state per range, merged.
    P = 8
    bounds = np.linspace(0, k.shape[0], P + 1).astype(int)
    qd = dev(q)
    ml = torch.empty((P, H, 2), dtype=torch.float32, device="cuda")
    acc = torch.empty((P, H, D), dtype=torch.float32, device="cuda")
    for r in range(P):
        kd, vd = dev(k[bounds[r]:bounds[r + 1]]), dev(v[bounds[r]:bounds[r + 1]])
        A.decode_attn_partial(qd, kd, vd, int(bounds[r + 1] - bounds[r]), ml[r], acc[r], H, Hkv, D)
    out = torch.empty_like(qd)
    A.lse_merge(ml, acc, P, out, H, D)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert_close(out.cpu().numpy(), exact, what="cfg4 partial+merge")
    # the states themselves against the oracle's (m in log2 units)
    m0, l0, a0 = O.partial_f64(q, k, v, int(bounds[0]), int(bounds[1]))
    mlh = ml.cpu().numpy()
    assert np.allclose(mlh[0, :, 0], m0, rtol=1e-5, atol=1e-4)
    sc = np.exp2(m0 - mlh[0, :, 0])          # rescale in case the maxima differ in rounding
    assert np.allclose(mlh[0, :, 1], l0 * sc, rtol=1e-4)


def test_partial_empty_range():
    q = W.normal_fp16(np.random.default_rng(1), (8, 64))
    ml = torch.empty((8, 2), dtype=torch.float32, device="cuda")
    acc = torch.empty((8, 64), dtype=torch.float32, device="cuda")
    A.decode_attn_partial(dev(q), 0, 0, 0, ml, acc, 8, 2, 64)
    torch.cuda.synchronize()
    m = ml.cpu().numpy()
    assert np.all(np.isneginf(m[:, 0])) and np.all(m[:, 1] == 0) and torch.all(acc == 0)


def test_prefill_golden_and_random():
    from pathlib import Path
    z = np.load(Path(__file__).parent / "golden" / "prefill_t37_h14_kv2_d64.npz")
    q, k, v = z["q"], z["k"], z["v"]
    T, H, D = q.shape
    out = nan_like(dev(q))
    A.prefill_attn_causal(dev(q), dev(k), dev(v), out, T, H, k.shape[1], D)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), z["exact"], what="prefill golden")
    rng = np.random.default_rng(77)
    T, H, Hkv, D = 300, 12, 2, 128
    q = W.normal_fp16(rng, (T, H, D))
    k = W.normal_fp16(rng, (T, Hkv, D))
    v = W.normal_fp16(rng, (T, Hkv, D))
    out = nan_like(dev(q))
    A.prefill_attn_causal(dev(q), dev(k), dev(v), out, T, H, Hkv, D)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), O.prefill_f64(q, k, v), what="prefill T300")


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("H,Hkv", [(14, 2), (28, 4), (8, 8), (32, 2)])
@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 129, 700])
def test_prefill_shapes_and_lengths(D, H, Hkv, T):
    """Causal prefill across query-tile boundaries (64 rows), partial last
    tiles and GQA groups of 1 to 16 heads."""
    q, k, v = (W.normal_fp16(np.random.default_rng([T, H, Hkv, D, i]), (T, n, D))
               for i, n in enumerate((H, Hkv, Hkv)))
    out = nan_like(dev(q))
    A.prefill_attn_causal(dev(q), dev(k), dev(v), out, T, H, Hkv, D)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert_close(out.cpu().numpy(), O.prefill_f64(q, k, v), what=f"prefill T{T} H{H} Hkv{Hkv} D{D}")


def test_rope_append_matches_oracle():
    rng = np.random.default_rng(8)
    H, Hkv, D, S, pos = 12, 2, 128, 600, 511
    q = W.normal_fp16(rng, (1, H, D))
    k = W.normal_fp16(rng, (1, Hkv, D))
    v = W.normal_fp16(rng, (1, Hkv, D))
    kc = W.normal_fp16(rng, (S, Hkv, D))
    vc = W.normal_fp16(rng, (S, Hkv, D))
    cos_d, sin_d = A.rope_precompute_tables(S, D, W.ROPE_THETA)
    ct, st = O.c_rope_tables(S, D, W.ROPE_THETA)
    assert np.array_equal(cos_d.cpu().numpy(), ct) and np.array_equal(sin_d.cpu().numpy(), st)
    qd, kd, vd, kcd, vcd = dev(q), dev(k), dev(v), dev(kc), dev(vc)
    A.rope_append(qd, kd, vd, kcd, vcd, cos_d, sin_d, 1, H, Hkv, D, pos)
    torch.cuda.synchronize()
    qo, ko, kco, vco = O.c_rope_append(q, k, v, kc, vc, ct, st, pos)
    # one fp16 ulp: the GPU may contract a*c - b*s into an FMA
    for got, want, what in [(qd, qo, "q"), (kd, ko, "k"), (kcd, kco, "k_cache"), (vcd, vco, "v_cache")]:
        g = got.cpu().numpy().astype(np.float64)
        w = want.astype(np.float64)
        assert np.all(np.abs(g - w) <= np.abs(w) * 2 ** -10 + 1e-7), what
    assert np.array_equal(vcd.cpu().numpy(), vco)


@pytest.mark.parametrize("H,Hkv,D,T", [(28, 4, 128, 50000), (12, 2, 128, 77777),
                                       (14, 2, 64, 200003), (28, 4, 128, 131072)])
def test_long_single_sequence_repeated_and_replayed(H, Hkv, D, T):
    """Long single sequences (many tiles per CTA, several clusters per kv
    head): eager calls in a row, then CUDA-graph replays of three calls with
    launch overlap on; the merge counters must be back at zero after every
    call."""
    q, k, v = W.decode_inputs(200 + T % 97, H, Hkv, D, T)
    exact = O.decode_f64(q, k, v)
    qd, kd, vd = dev(q), dev(k), dev(v)
    lib = A.load()
    s = torch.cuda.Stream()
    out = nan_like(qd)
    for _ in range(3):
        out.fill_(float("nan"))
        with torch.cuda.stream(s):
            A.decode_attn_v4_flash(qd, kd, vd, out, H, Hkv, D, T, s)
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert_close(out.cpu().numpy(), exact, what=f"long eager T={T}")
    outs = [nan_like(qd) for _ in range(3)]
    lib.fr_set_launch_overlap(1)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for o in outs:
                A.decode_attn_v4_flash(qd, kd, vd, o, H, Hkv, D, T, s)
        for _ in range(3):
            for o in outs:
                o.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert A.device_error() == 0
            for o in outs:
                assert_close(o.cpu().numpy(), exact, what=f"long graph T={T}")
    finally:
        lib.fr_set_launch_overlap(0)


@pytest.mark.parametrize("T,H,Hkv,D,which", [(1, 14, 2, 64, "qkv"), (5, 12, 2, 128, "qkv"),
                                             (1, 28, 4, 128, "q"), (3, 8, 8, 64, "kv")])
def test_qkv_bias_rope_append_matches_oracle(T, H, Hkv, D, which):
    rng = np.random.default_rng(9 + T + D)
    S, pos = 300, 200
    q = W.normal_fp16(rng, (T, H, D))
    k = W.normal_fp16(rng, (T, Hkv, D))
    v = W.normal_fp16(rng, (T, Hkv, D))
    biases = [W.normal_fp16(rng, (n * D,)) if c in which else None
              for n, c in ((H, "q"), (Hkv, "k"), (Hkv, "v"))]
    kc = W.normal_fp16(rng, (S, Hkv, D))
    vc = W.normal_fp16(rng, (S, Hkv, D))
    cos_d, sin_d = A.rope_precompute_tables(S, D, W.ROPE_THETA)
    ct, st = O.c_rope_tables(S, D, W.ROPE_THETA)
    qd, kd, vd, kcd, vcd = dev(q), dev(k), dev(v), dev(kc), dev(vc)
    bd = [None if b is None else dev(b) for b in biases]
    A.qkv_bias_rope_append(qd, kd, vd, bd[0], bd[1], bd[2], kcd, vcd, cos_d, sin_d, T, H, Hkv, D,
                           pos)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    qo, ko, vo, kco, vco = O.c_qkv_bias_rope_append(q, k, v, *biases, kc, vc, ct, st, pos)
    # one fp16 ulp where the rotation is involved (FMA contraction of a*c - b*s)
    for got, want, what in [(qd, qo, "q"), (kd, ko, "k"), (kcd, kco, "k_cache")]:
        g = got.cpu().numpy().astype(np.float64)
        w = want.astype(np.float64)
        assert np.all(np.abs(g - w) <= np.abs(w) * 2 ** -10 + 1e-7), what
    # the bias add alone is exact
    assert np.array_equal(vd.cpu().numpy().view(np.uint16), vo.view(np.uint16))
    assert np.array_equal(vcd.cpu().numpy().view(np.uint16), vco.view(np.uint16))


def test_against_reference_gpu_kernel():
    ref = O.load_ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    for q, k, v in [W.cfg1_inputs(), W.decode_inputs(3, 12, 2, 128, 4096)]:
        H, D = q.shape
        Hkv = k.shape[1]
        qd, kd, vd = dev(q), dev(k), dev(v)
        out_ref = nan_like(qd)
        ref.ref_decode_attn_v4_flash(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                     out_ref.data_ptr(), H, Hkv, D, k.shape[0], None)
        torch.cuda.synchronize()
        exact = O.decode_f64(q, k, v)
        ours = decode(q, k, v)
        assert_close(out_ref.cpu().numpy(), exact, what="reference v4 vs exact")
        assert_close(ours, out_ref.cpu().numpy(), what="ours vs reference v4")


def test_graph_capture_replay():
    q, k, v = W.decode_inputs(11, 12, 2, 128, 8192)
    H, D = q.shape
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = nan_like(qd)
    A.reserve_workspace(A.decode_workspace_size(1, H, 2, D, 8192))
    A.decode_attn_v4_flash(qd, kd, vd, out, H, 2, D, 8192)     # first call outside capture
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    out.fill_(float("nan"))
    with torch.cuda.graph(g, stream=s):
        A.decode_attn_v4_flash(qd, kd, vd, out, H, 2, D, 8192, stream=torch.cuda.current_stream())
    g.replay()
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), O.decode_f64(q, k, v), what="graph replay")


def test_invalid_arguments_raise():
    qd = torch.zeros((8, 64), dtype=torch.float16, device="cuda")
    kd = torch.zeros((16, 2, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(ForgeRTError) as e:
        A.decode_attn_v4_flash(qd, kd, kd, qd, 8, 3, 64, 16)     # 8 % 3 != 0
    assert e.value.status == 1
    with pytest.raises(ForgeRTError) as e:
        A.decode_attn_v4_flash(qd, kd, kd, qd, 8, 2, 96, 16)     # unsupported head_dim
    assert e.value.status == 2
    with pytest.raises(ForgeRTError) as e:
        A.decode_attn_v4_flash(qd, kd.data_ptr() + 2, kd, qd, 8, 2, 64, 16)  # misaligned k
    assert e.value.status == 3
    with pytest.raises(ForgeRTError) as e:
        A.decode_attn_v4_flash(qd, kd, kd, qd, 8, 2, 64, 0)      # empty cache
    assert e.value.status == 1
    assert A.device_error() == 0


@pytest.mark.parametrize("use_graph", [False, True])
def test_overlap_mode_after_rope_append(use_graph):
    """Decode step as the runtime runs it, on a non-default stream with launch
    overlap on: the fused prologue appends row kv_len-1 (and rotates q) right
    before each attention call, which may prefetch only the older rows
    before its grid-dependency wait.  Four layers back to back."""
    from forgert_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(17)
    L, H, Hkv, D, S, kv = 4, 12, 2, 128, 6000, 5000
    cos_d, sin_d = A.rope_precompute_tables(S, D, W.ROPE_THETA)
    ct, st = O.c_rope_tables(S, D, W.ROPE_THETA)
    caches = [(W.normal_fp16(rng, (S, Hkv, D)), W.normal_fp16(rng, (S, Hkv, D))) for _ in range(L)]
    qs = [W.normal_fp16(rng, (1, H, D)) for _ in range(L)]
    knew = [W.normal_fp16(rng, (1, Hkv, D)) for _ in range(L)]
    vnew = [W.normal_fp16(rng, (1, Hkv, D)) for _ in range(L)]
    dev_caches = [(dev(k), dev(v)) for k, v in caches]
    dq = [dev(q) for q in qs]
    dk = [dev(k) for k in knew]
    dv = [dev(v) for v in vnew]
    outs = [torch.full((H, D), float("nan"), dtype=torch.float16, device="cuda") for _ in range(L)]
    A.reserve_workspace(A.decode_workspace_size(1, H, Hkv, D, kv))
    s = torch.cuda.Stream()
    old = lib.fr_set_launch_overlap(1)
    try:
        def step(stream):
            for l in range(L):
                A.rope_append(dq[l], dk[l], dv[l], dev_caches[l][0], dev_caches[l][1], cos_d, sin_d,
                              1, H, Hkv, D, kv - 1, stream)
                A.decode_attn_v4_flash(dq[l], dev_caches[l][0], dev_caches[l][1], outs[l], H, Hkv,
                                       D, kv, stream)
        # warm once outside capture (library state), then restore the inputs
        with torch.cuda.stream(s):
            step(s)
        torch.cuda.synchronize()
        for l in range(L):
            dq[l].copy_(dev(qs[l]))
            dk[l].copy_(dev(knew[l]))
            outs[l].fill_(float("nan"))
        torch.cuda.synchronize()
        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                step(torch.cuda.current_stream())
            g.replay()
        else:
            with torch.cuda.stream(s):
                step(s)
        torch.cuda.synchronize()
    finally:
        lib.fr_set_launch_overlap(old)
    assert A.device_error() == 0
    for l in range(L):
        qo, ko, kco, vco = O.c_rope_append(qs[l], knew[l], vnew[l], caches[l][0], caches[l][1],
                                           ct, st, kv - 1)
        exact = O.decode_f64(qo[0], kco, vco, kv)
        assert_close(outs[l].cpu().numpy(), exact, what=f"overlap layer {l}")


_GROUPED_PROCESS = r"""
import json, sys
sys.path.insert(0, sys.argv[1])
import numpy as np, torch
from forgert_b200 import attention as A, _lib, workloads as W
lib = _lib.load()
lib.fr_set_launch_overlap(1)
s = torch.cuda.Stream()
outs = {}
for (H, Hkv, D, T) in json.loads(sys.argv[3]):
    rng = np.random.default_rng(T + 7 * H + D)
    q = W.normal_fp16(rng, (H, D)); k = W.normal_fp16(rng, (T, Hkv, D)); v = W.normal_fp16(rng, (T, Hkv, D))
    d = lambda a: torch.from_numpy(a).cuda()
    qd, kd, vd = d(q), d(k), d(v)
    out = torch.full_like(qd, float("nan"))
    with torch.cuda.stream(s):
        for _ in range(3):                       # chained calls (launch overlap on a stream)
            A.decode_attn_v4_flash(qd, kd, vd, out, H, Hkv, D, T, s)
    torch.cuda.synchronize()
    outs[f"{H}_{Hkv}_{D}_{T}"] = out.cpu().numpy()
np.savez(sys.argv[2], **outs)
print(json.dumps({"err": A.device_error()}))
"""

_GROUPED_CASES = [(12, 2, 128, 1025), (12, 2, 128, 2048), (12, 2, 128, 4096), (12, 2, 128, 4097),
                  (28, 4, 128, 3000), (14, 2, 64, 2048), (32, 2, 128, 4096), (40, 2, 64, 1500)]


@pytest.mark.parametrize("grouped", ["1", "0"])
def test_grouped_consumers(tmp_path, grouped):
    """Single-sequence calls of a few thousand positions run the kernel form
    with two consumer groups taking alternate tiles (FORGERT_GROUPED, read
    once per process, default on); with it off they run the four-warp form.
    Both match the oracle, on a stream with launch overlap, and the plan trace
    shows which form ran."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, FORGERT_GROUPED=grouped, FORGERT_TRACE_PLAN="1")
    f = tmp_path / "out.npz"
    r = subprocess.run([sys.executable, "-c", _GROUPED_PROCESS, str(root), str(f),
                        json.dumps(_GROUPED_CASES)], env=env, capture_output=True, text=True,
                       timeout=600, cwd=str(root))
    assert r.returncode == 0, r.stderr[-3000:]
    assert json.loads(r.stdout.strip().splitlines()[-1])["err"] == 0
    plans = [ln for ln in r.stderr.splitlines() if "[forgert] plan" in ln]
    assert plans and any(f"grouped={grouped}" in ln for ln in plans)
    if grouped == "0":
        assert not any("grouped=1" in ln for ln in plans)
    outs = np.load(f)
    for (H, Hkv, D, T) in _GROUPED_CASES:
        rng = np.random.default_rng(T + 7 * H + D)
        q = W.normal_fp16(rng, (H, D))
        k = W.normal_fp16(rng, (T, Hkv, D))
        v = W.normal_fp16(rng, (T, Hkv, D))
        assert_close(outs[f"{H}_{Hkv}_{D}_{T}"], O.decode_f64(q, k, v),
                     what=f"grouped={grouped} H{H} Hkv{Hkv} D{D} T{T}")
