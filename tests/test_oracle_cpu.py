"""Pins the CPU oracle (no GPU needed).

The C restatement must reproduce the reference's own cpu_decode_attn
(tests/test_kernels.cpp:229-270) bit for bit: against the committed golden
vectors (made by running the reference code, tests/golden/make_golden.py)
and, where oracle/_ref was built from the reference sources, live on fresh
random cases.  The fp64 oracles must agree with each other and with the
reference to fp32 rounding.
"""
from __future__ import annotations

import ast
from pathlib import Path

import numpy as np
import pytest

from forgert_b200 import workloads as W
from oracle import oracle as O

GOLD = Path(__file__).parent / "golden"
WITH_INPUTS = ["ref_h8_kv2_d64_len128", "ref_h8_kv2_d64_len1", "ref_h8_kv2_d128_len128",
               "gqa7_d128_len33", "gqa16_d64_len200", "mha_d128_len100", "gqa6_d128_len300"]


def load(name):
    z = np.load(GOLD / f"{name}.npz")
    meta = ast.literal_eval(str(z["meta"])) if "meta" in z.files else {}
    return z, meta


def f32(*a):
    return [x.astype(np.float32) for x in a]


@pytest.mark.parametrize("name", WITH_INPUTS)
def test_c_restatement_bit_exact_vs_reference_golden(name):
    z, meta = load(name)
    q, k, v = z["q"], z["k"], z["v"]
    assert meta["inputs_sha256"] == __import__("hashlib").sha256(
        q.tobytes() + k.tobytes() + v.tobytes()).hexdigest()
    out = O.c_decode_f32(*f32(q, k, v))
    assert np.array_equal(out, z["ref_f32"])


def test_cfg1_regenerates_and_matches_reference_golden():
    z, meta = load("cfg1_h14_kv2_d64_len512")
    q, k, v = W.cfg1_inputs()
    import hashlib
    assert hashlib.sha256(q.tobytes() + k.tobytes() + v.tobytes()).hexdigest() == meta["inputs_sha256"]
    assert np.array_equal(O.c_decode_f32(*f32(q, k, v)), z["ref_f32"])
    assert np.allclose(O.decode_f64(q, k, v), z["exact"], rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", WITH_INPUTS)
def test_fp64_oracles_agree(name):
    z, _ = load(name)
    q, k, v = z["q"], z["k"], z["v"]
    np_out = O.decode_f64(q, k, v)
    c_out = O.c_decode_f64(q, k, v)
    assert np.allclose(np_out, z["exact"], rtol=0, atol=1e-12)
    assert np.allclose(c_out, np_out, rtol=0, atol=1e-12)
    # the reference's fp32 oracle sits within fp32 rounding of the exact value
    a, _ = O.max_errors(z["ref_f32"], np_out)
    assert a < 5e-6


@pytest.mark.parametrize("name", WITH_INPUTS)
def test_hf_eager_fixture_within_fp16_probability_rounding(name):
    """transformers' eager attention (python/reference.py's arithmetic) rounds
    probabilities to fp16; it stays within the spec's absolute tolerance."""
    z, _ = load(name)
    a, _ = O.max_errors(z["hf_f16"], z["exact"])
    assert a <= 2e-3


def test_live_reference_bit_exact():
    if O.load_ref() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    rng = np.random.default_rng(99)
    for H, Hkv, D, T in [(8, 2, 64, 1), (14, 2, 64, 77), (28, 4, 128, 129), (4, 4, 128, 300),
                         (32, 2, 64, 65), (12, 2, 128, 1000)]:
        q = rng.uniform(-1, 1, (H, D)).astype(np.float32)
        k = rng.standard_normal((T, Hkv, D)).astype(np.float32)
        v = rng.standard_normal((T, Hkv, D)).astype(np.float32)
        assert np.array_equal(O.c_decode_f32(q, k, v), O.ref_cpu_decode_attn(q, k, v)), (H, Hkv, D, T)


def test_partial_merge_algebra():
    q, k, v = W.decode_inputs(4, 28, 4, 128, 1000)
    exact = O.decode_f64(q, k, v)
    bounds = [0, 0, 130, 131, 640, 1000, 1000]      # includes empty ranges
    parts = [O.partial_f64(q, k, v, bounds[i], bounds[i + 1]) for i in range(len(bounds) - 1)]
    m = np.stack([p[0] for p in parts])
    l = np.stack([p[1] for p in parts])
    acc = np.stack([p[2] for p in parts])
    assert np.allclose(O.merge_f64(m, l, acc), exact, rtol=0, atol=1e-12)
    assert np.allclose(O.c_merge_f64(m, l, acc), exact, rtol=0, atol=1e-12)
    cm, cl, ca = O.c_partial_f64(q, k, v, 130, 640)
    nm, nl, na = O.partial_f64(q, k, v, 130, 640)
    assert np.allclose(cm, nm, atol=1e-12) and np.allclose(cl, nl, rtol=1e-12)
    assert np.allclose(ca, na, rtol=1e-12, atol=1e-12)
    # all-empty merge gives zeros, no NaN
    e = O.partial_f64(q, k, v, 5, 5)
    z = O.merge_f64(e[0][None], e[1][None], e[2][None])
    assert np.all(z == 0)


def test_prefill_oracles():
    z = np.load(GOLD / "prefill_t37_h14_kv2_d64.npz")
    q, k, v = z["q"], z["k"], z["v"]
    np_out = O.prefill_f64(q, k, v)
    assert np.allclose(np_out, z["exact"], atol=1e-12)
    assert np.allclose(O.c_prefill_f64(q, k, v), np_out, atol=1e-12)
    a, _ = O.max_errors(z["hf_f16"], np_out)
    assert a <= 2e-3
    # row s of causal prefill is a decode over the first s+1 positions
    for s in (0, 1, 17, 36):
        assert np.allclose(np_out[s], O.decode_f64(q[s], k[:s + 1], v[:s + 1]), atol=1e-12)


def test_rope_oracles():
    c1, s1 = O.c_rope_tables(512, 64, W.ROPE_THETA)
    c2, s2 = O.rope_tables_f64(512, 64, W.ROPE_THETA)
    # both evaluate in fp64 and round once to fp32: equal up to libm's last double ulp
    assert np.max(np.abs(c1 - c2)) <= 6e-8 and np.max(np.abs(s1 - s2)) <= 6e-8
    assert np.all(c1[0] == 1) and np.all(s1[0] == 0)
    z = np.load(GOLD / "rope_d64_pos40.npz")
    x = z["x"]
    ct, st = O.c_rope_tables(64, 64, float(z["theta"]))
    ours = O.rope_apply(x, ct, st, 40)
    # transformers rounds cos/sin to fp16 before rotating (fp16 products);
    # the reference (and this oracle) keep fp32 tables and fp32 products.
    assert np.max(np.abs(ours.astype(np.float64) - z["hf_f16"].astype(np.float64))) <= 8e-3
    # C and numpy restatements agree bit for bit
    T, Hh, D = x.shape
    kc = np.zeros((64, 2, D), np.float16)
    qo, ko, kco, vco = O.c_rope_append(x, x[:, :2].copy(), x[:, :2].copy(), kc, kc, ct, st, 40)
    assert np.array_equal(qo, ours)
    assert np.array_equal(kco[40:44], ours[:, :2]) and np.array_equal(vco[40:44], x[:, :2])


def test_half_conversion_bit_exact():
    lib = O.load_oracle()
    rng = np.random.default_rng(3)
    vals = np.concatenate([
        rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 5, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 5.96e-8, 2.98e-8, 2.99e-8,
                  6.1035e-5, 6.103515625e-05, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11]),
    ])
    with np.errstate(over="ignore"):
        for x in vals:
            got = lib.oracle_double_to_half(float(x))
            want = np.array([x], np.float64).astype(np.float16).view(np.uint16)[0]
            assert got == want, (x, hex(got), hex(want))
            assert lib.oracle_half_to_float(int(want)) == np.float32(np.float16(x))


def test_paged_layout_round_trip():
    """paginate() + paged_f64 (gather by block table) reproduce the contiguous
    per-sequence caches exactly, whatever order the pages were handed out in."""
    rng = np.random.default_rng(21)
    lens = np.array([1, 15, 16, 17, 100, 0, 64], np.int32)
    ks = [W.normal_fp16(rng, (int(n), 2, 64)) for n in lens]
    vs = [W.normal_fp16(rng, (int(n), 2, 64)) for n in lens]
    q = W.normal_fp16(rng, (len(lens), 8, 64))
    for page in (16, 48):
        kp, vp, table = W.paginate(ks, vs, page, seed=page, spare_pages=3)
        assert np.isnan(kp.astype(np.float32)).any()          # unowned rows are NaN
        for b, n in enumerate(lens):
            t = np.arange(int(n))
            assert np.array_equal(kp[table[b, t // page], t % page], ks[b])
            assert (table[b, -(-int(n) // page):] == -1).all()
        assert np.array_equal(O.paged_f64(q, kp, vp, table, lens, page),
                              O.batched_f64(q, ks, vs, lens))


def test_bias_prologue_oracle():
    """q/k/v bias add is one fp16 RN addition (numpy's float16 add rounds the
    exact sum once, as __hadd does); with no biases the prologue is exactly
    the RoPE + append oracle."""
    rng = np.random.default_rng(31)
    T, H, Hkv, D, S, pos = 3, 14, 2, 64, 40, 30
    q = W.normal_fp16(rng, (T, H, D))
    k = W.normal_fp16(rng, (T, Hkv, D))
    v = W.normal_fp16(rng, (T, Hkv, D))
    bq = W.normal_fp16(rng, (H * D,))
    bk = W.normal_fp16(rng, (Hkv * D,))
    bv = W.normal_fp16(rng, (Hkv * D,))
    kc = W.normal_fp16(rng, (S, Hkv, D))
    vc = W.normal_fp16(rng, (S, Hkv, D))
    ct, st = O.c_rope_tables(S, D, W.ROPE_THETA)
    got = O.c_qkv_bias_rope_append(q, k, v, bq, bk, bv, kc, vc, ct, st, pos)
    qb = (q + bq.reshape(H, D)).astype(np.float16)
    kb = (k + bk.reshape(Hkv, D)).astype(np.float16)
    vb = (v + bv.reshape(Hkv, D)).astype(np.float16)
    want = O.c_rope_append(qb, kb, vb, kc, vc, ct, st, pos)
    for g, w in zip((got[0], got[1], got[3], got[4]), want):
        assert np.array_equal(g.view(np.uint16), w.view(np.uint16))
    assert np.array_equal(got[2].view(np.uint16), vb.view(np.uint16))
    plain = O.c_qkv_bias_rope_append(q, k, v, None, None, None, kc, vc, ct, st, pos)
    ref = O.c_rope_append(q, k, v, kc, vc, ct, st, pos)
    for g, w in zip((plain[0], plain[1], plain[3], plain[4]), ref):
        assert np.array_equal(g.view(np.uint16), w.view(np.uint16))
