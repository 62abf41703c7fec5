"""CPU oracle for the decode-attention path.

TEST INFRASTRUCTURE ONLY: this module is the parity checker.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference arms may
import it; the product package (forgert_b200) never does.

Three oracles, all on the CPU:
  * numpy fp64 restatements (this file) - fast enough for every benchmark
    size; the exact values fp16 outputs are compared against.
  * liboracle.so (decode_attn_oracle.c) - the C restatement, including
    oracle_decode_attn_f32, an operation-for-operation restatement of the
    reference's cpu_decode_attn (tests/test_kernels.cpp:229-270).
  * libforgert_ref.so (oracle/_ref, built from the reference sources by
    oracle/Makefile) - the reference's own cpu_decode_attn and its GPU
    kernels, used to pin the restatements.

Shapes follow the reference: q [H, D], cache views [T, Hkv, D], query head h
reads kv head h // (H // Hkv).
"""
from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libforgert_ref.so"
LOG2E = 1.4426950408889634

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ct)


# ---------------------------------------------------------------- loaders
_oracle_lib = None
_ref_lib = None


def load_oracle() -> ctypes.CDLL:
    """The C restatement; built with `make -C oracle` if it is missing."""
    global _oracle_lib
    if _oracle_lib is None:
        if not ORACLE_LIB.exists():
            subprocess.run(["make", "-C", str(HERE), str(ORACLE_LIB)], check=True,
                           capture_output=True)
        lib = ctypes.CDLL(str(ORACLE_LIB))
        lib.oracle_decode_attn_f32.argtypes = [_f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 4
        lib.oracle_decode_attn_f64.argtypes = [_u16p, _u16p, _u16p, _f64p] + [ctypes.c_int] * 4
        lib.oracle_partial_f64.argtypes = [_u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_int,
                                           _f64p, _f64p, _f64p] + [ctypes.c_int] * 3
        lib.oracle_merge_f64.argtypes = [_f64p, _f64p, _f64p, ctypes.c_int, _f64p,
                                         ctypes.c_int, ctypes.c_int]
        lib.oracle_prefill_f64.argtypes = [_u16p, _u16p, _u16p, _f64p] + [ctypes.c_int] * 4
        lib.oracle_rope_tables_f64.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_double, ctypes.c_double]
        lib.oracle_rope_append.argtypes = [_u16p, _u16p, _u16p, _u16p, _u16p, _f32p, _f32p] + \
            [ctypes.c_int] * 5
        lib.oracle_qkv_bias_rope_append.argtypes = [_u16p] * 8 + [_f32p, _f32p] + \
            [ctypes.c_int] * 5
        lib.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        lib.oracle_half_to_float.restype = ctypes.c_float
        lib.oracle_double_to_half.argtypes = [ctypes.c_double]
        lib.oracle_double_to_half.restype = ctypes.c_uint16
        _oracle_lib = lib
    return _oracle_lib


def load_ref() -> ctypes.CDLL | None:
    """The reference's own code (oracle/_ref), or None where it was not built."""
    global _ref_lib
    if _ref_lib is None and REF_LIB.exists():
        lib = ctypes.CDLL(str(REF_LIB))
        lib.ref_cpu_decode_attn.argtypes = [_f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 4
        pp = ctypes.POINTER(_f32p)
        lib.ref_cpu_decode_attn_many.argtypes = [pp, pp, pp, pp, ctypes.POINTER(ctypes.c_int)] + \
            [ctypes.c_int] * 5
        vp = ctypes.c_void_p
        lib.ref_decode_attn_v4_flash.argtypes = [vp, vp, vp, vp] + [ctypes.c_int] * 4 + [vp]
        lib.ref_prefill_attn_causal.argtypes = [vp, vp, vp, vp] + [ctypes.c_int] * 4 + [vp]
        lib.ref_rope_v2_fused.argtypes = [vp, vp, vp, vp] + [ctypes.c_int] * 5 + [vp]
        lib.ref_bias_add_broadcast.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, vp]
        lib.ref_rope_precompute_tables.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_float, ctypes.c_float]
        lib.ref_rope_precompute_tables.restype = ctypes.c_int
        lib.ref_run_kernel_tests.restype = ctypes.c_int
        _ref_lib = lib
    return _ref_lib


# ------------------------------------------------------- numpy fp64 oracles
def _as_f64(x: np.ndarray) -> np.ndarray:
    return np.asarray(x).astype(np.float64)


def decode_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_len: int | None = None) -> np.ndarray:
    """Exact decode attention (cpu_decode_attn in fp64).

    q: [H, D] fp16; k, v: [>= kv_len, Hkv, D] fp16.  Returns [H, D] float64.
    An empty range (kv_len == 0) yields zeros.
    """
    H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    T = k.shape[0] if kv_len is None else kv_len
    out = np.zeros((H, D), np.float64)
    if T == 0:
        return out
    scale = 1.0 / math.sqrt(D)
    qf = _as_f64(q).reshape(Hkv, G, D)
    for h in range(Hkv):
        kf = _as_f64(k[:T, h, :])                  # [T, D]
        vf = _as_f64(v[:T, h, :])
        s = qf[h] @ kf.T * scale                   # [G, T]
        s -= s.max(axis=1, keepdims=True)
        e = np.exp(s)
        out[h * G:(h + 1) * G] = (e @ vf) / e.sum(axis=1, keepdims=True)
    return out


def decode_f64_fp16_probs(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """HF eager semantics (transformers Qwen2 eager_attention_forward): the
    fp32 softmax is rounded to fp16 before the P.V product."""
    H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    out = np.zeros((H, D), np.float64)
    qf = _as_f64(q).reshape(Hkv, G, D)
    for h in range(Hkv):
        kf = _as_f64(k[:, h, :])
        vf = _as_f64(v[:, h, :])
        s = (qf[h] @ kf.T / math.sqrt(D)).astype(np.float32)
        s = s - s.max(axis=1, keepdims=True)
        e = np.exp(s)
        p = (e / e.sum(axis=1, keepdims=True)).astype(np.float16).astype(np.float64)
        out[h * G:(h + 1) * G] = p @ vf
    return out


def batched_f64(q: np.ndarray, ks: list, vs: list, lens) -> np.ndarray:
    """q: [B, H, D]; ks[b], vs[b]: [>= lens[b], Hkv, D]."""
    return np.stack([decode_f64(q[b], ks[b], vs[b], int(lens[b])) for b in range(q.shape[0])])


def paged_f64(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray, block_table: np.ndarray,
              lens, page_size: int) -> np.ndarray:
    """Paged cache [num_pages, page_size, Hkv, D]: sequence b's position t is
    row t % page_size of page block_table[b, t // page_size].  The rows are
    gathered back into one contiguous cache per sequence (the reference's
    layer-view layout, runtime/kv_cache.cpp:29-37) and decoded with
    batched_f64."""
    ks, vs = [], []
    for b, n in enumerate(lens):
        n = int(n)
        t = np.arange(n)
        pages = block_table[b, t // page_size]
        ks.append(k_pages[pages, t % page_size])
        vs.append(v_pages[pages, t % page_size])
    return batched_f64(q, ks, vs, lens)


def partial_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, begin: int, end: int):
    """(m, l, acc) over positions [begin, end), base 2: m = max_t s_t log2(e)/sqrt(D)."""
    H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    m = np.full(H, -np.inf)
    l = np.zeros(H)
    acc = np.zeros((H, D))
    if end <= begin:
        return m, l, acc
    qf = _as_f64(q).reshape(Hkv, G, D)
    sl2 = LOG2E / math.sqrt(D)
    for h in range(Hkv):
        kf = _as_f64(k[begin:end, h, :])
        vf = _as_f64(v[begin:end, h, :])
        s2 = qf[h] @ kf.T * sl2
        mh = s2.max(axis=1)
        w = np.exp2(s2 - mh[:, None])
        m[h * G:(h + 1) * G] = mh
        l[h * G:(h + 1) * G] = w.sum(axis=1)
        acc[h * G:(h + 1) * G] = w @ vf
    return m, l, acc


def merge_f64(m: np.ndarray, l: np.ndarray, acc: np.ndarray) -> np.ndarray:
    """m, l: [S, H]; acc: [S, H, D] -> normalised output [H, D]."""
    mx = m.max(axis=0)
    mu = np.where(np.isinf(mx), 0.0, mx)
    w = np.exp2(m - mu[None])
    lt = (l * w).sum(axis=0)
    num = (acc * w[:, :, None]).sum(axis=0)
    return np.where(lt[:, None] > 0, num / np.where(lt > 0, lt, 1.0)[:, None], 0.0)


def prefill_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Causal: q [T, H, D], k/v [T, Hkv, D]; position s sees 0..s."""
    T, H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    out = np.zeros((T, H, D))
    qf = _as_f64(q)
    mask = np.triu(np.full((T, T), -np.inf), 1)
    for h in range(Hkv):
        kf = _as_f64(k[:, h, :])
        vf = _as_f64(v[:, h, :])
        for g in range(G):
            s = qf[:, h * G + g, :] @ kf.T / math.sqrt(D) + mask
            s -= s.max(axis=1, keepdims=True)
            e = np.exp(s)
            out[:, h * G + g, :] = (e @ vf) / e.sum(axis=1, keepdims=True)
    return out


def rope_tables_f64(max_seq_len: int, head_dim: int, base: float, scale: float = 1.0):
    """cos/sin [max_seq_len, D/2] fp32 of theta = pos / (base^(2f/D) * scale)."""
    f = np.arange(head_dim // 2, dtype=np.float64)
    inv = 1.0 / (np.power(float(base), 2.0 * f / head_dim) * scale)
    th = np.arange(max_seq_len, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)


def rope_apply(x: np.ndarray, cos_t: np.ndarray, sin_t: np.ndarray, pos_offset: int) -> np.ndarray:
    """NeoX rotation of x [T, heads, D] fp16 (fp32 math, fp16 result),
    kernels/rope.cu:180-190."""
    T, _, D = x.shape
    hd = D // 2
    xf = x.astype(np.float32)
    pos = np.arange(T) + pos_offset
    c = cos_t[pos][:, None, :]
    s = sin_t[pos][:, None, :]
    a, b = xf[..., :hd], xf[..., hd:]
    return np.concatenate([a * c - b * s, a * s + b * c], axis=-1).astype(np.float16)


# --------------------------------------------------------- C entry points
def c_decode_f32(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """The C restatement of cpu_decode_attn (fp32 in, fp32 out)."""
    lib = load_oracle()
    H, D = q.shape
    T, Hkv, _ = k.shape
    qf, kf, vf = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    out = np.zeros((H, D), np.float32)
    lib.oracle_decode_attn_f32(_ptr(qf, _f32p), _ptr(kf, _f32p), _ptr(vf, _f32p),
                               _ptr(out, _f32p), H, Hkv, D, T)
    return out


def c_decode_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    lib = load_oracle()
    H, D = q.shape
    T, Hkv, _ = k.shape
    qh, kh, vh = (np.ascontiguousarray(a, dtype=np.float16).view(np.uint16) for a in (q, k, v))
    out = np.zeros((H, D), np.float64)
    lib.oracle_decode_attn_f64(_ptr(qh, _u16p), _ptr(kh, _u16p), _ptr(vh, _u16p),
                               _ptr(out, _f64p), H, Hkv, D, T)
    return out


def c_prefill_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    lib = load_oracle()
    T, H, D = q.shape
    Hkv = k.shape[1]
    qh, kh, vh = (np.ascontiguousarray(a, dtype=np.float16).view(np.uint16) for a in (q, k, v))
    out = np.zeros((T, H, D), np.float64)
    lib.oracle_prefill_f64(_ptr(qh, _u16p), _ptr(kh, _u16p), _ptr(vh, _u16p), _ptr(out, _f64p),
                           T, H, Hkv, D)
    return out


def c_partial_f64(q, k, v, begin: int, end: int):
    lib = load_oracle()
    H, D = q.shape
    Hkv = k.shape[1]
    qh, kh, vh = (np.ascontiguousarray(a, dtype=np.float16).view(np.uint16) for a in (q, k, v))
    m = np.zeros(H)
    l = np.zeros(H)
    acc = np.zeros((H, D))
    lib.oracle_partial_f64(_ptr(qh, _u16p), _ptr(kh, _u16p), _ptr(vh, _u16p), begin, end,
                           _ptr(m, _f64p), _ptr(l, _f64p), _ptr(acc, _f64p), H, Hkv, D)
    return m, l, acc


def c_merge_f64(m: np.ndarray, l: np.ndarray, acc: np.ndarray) -> np.ndarray:
    lib = load_oracle()
    S, H = m.shape
    D = acc.shape[2]
    m, l, acc = (np.ascontiguousarray(a, dtype=np.float64) for a in (m, l, acc))
    out = np.zeros((H, D))
    lib.oracle_merge_f64(_ptr(m, _f64p), _ptr(l, _f64p), _ptr(acc, _f64p), S, _ptr(out, _f64p),
                         H, D)
    return out


def c_rope_tables(max_seq_len: int, head_dim: int, base: float, scale: float = 1.0):
    lib = load_oracle()
    c = np.zeros((max_seq_len, head_dim // 2), np.float32)
    s = np.zeros_like(c)
    lib.oracle_rope_tables_f64(_ptr(c, _f32p), _ptr(s, _f32p), max_seq_len, head_dim, base, scale)
    return c, s


def c_rope_append(q, k, v, k_cache, v_cache, cos_t, sin_t, pos_offset: int):
    """Returns rotated (q, k) and updated (k_cache, v_cache) copies (fp16)."""
    lib = load_oracle()
    T, H, D = q.shape
    Hkv = k.shape[1]
    qh = np.ascontiguousarray(q, np.float16).copy().view(np.uint16)
    kh = np.ascontiguousarray(k, np.float16).copy().view(np.uint16)
    vh = np.ascontiguousarray(v, np.float16).view(np.uint16)
    kc = np.ascontiguousarray(k_cache, np.float16).copy().view(np.uint16)
    vc = np.ascontiguousarray(v_cache, np.float16).copy().view(np.uint16)
    ct = np.ascontiguousarray(cos_t, np.float32)
    st = np.ascontiguousarray(sin_t, np.float32)
    lib.oracle_rope_append(_ptr(qh, _u16p), _ptr(kh, _u16p), _ptr(vh, _u16p), _ptr(kc, _u16p),
                           _ptr(vc, _u16p), _ptr(ct, _f32p), _ptr(st, _f32p), T, H, Hkv, D,
                           pos_offset)
    return (qh.view(np.float16), kh.view(np.float16), kc.view(np.float16), vc.view(np.float16))


def c_qkv_bias_rope_append(q, k, v, q_bias, k_bias, v_bias, k_cache, v_cache, cos_t, sin_t,
                           pos_offset: int):
    """Biased + rotated (q, k), biased v and updated (k_cache, v_cache) copies
    (fp16); a None bias is skipped."""
    lib = load_oracle()
    T, H, D = q.shape
    Hkv = k.shape[1]
    bufs = [np.ascontiguousarray(a, np.float16).copy().view(np.uint16)
            for a in (q, k, v, k_cache, v_cache)]
    qh, kh, vh, kc, vc = bufs
    bias = [None if b is None else np.ascontiguousarray(b, np.float16).view(np.uint16)
            for b in (q_bias, k_bias, v_bias)]
    bp = [None if b is None else _ptr(b, _u16p) for b in bias]
    ct = np.ascontiguousarray(cos_t, np.float32)
    st = np.ascontiguousarray(sin_t, np.float32)
    lib.oracle_qkv_bias_rope_append(_ptr(qh, _u16p), _ptr(kh, _u16p), _ptr(vh, _u16p), bp[0],
                                    bp[1], bp[2], _ptr(kc, _u16p), _ptr(vc, _u16p),
                                    _ptr(ct, _f32p), _ptr(st, _f32p), T, H, Hkv, D, pos_offset)
    return tuple(b.view(np.float16) for b in (qh, kh, vh, kc, vc))


def ref_cpu_decode_attn(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """The reference's own cpu_decode_attn (needs oracle/_ref)."""
    lib = load_ref()
    if lib is None:
        raise FileNotFoundError(f"{REF_LIB} not built (make -C oracle REF=<reference tree>)")
    H, D = q.shape
    T, Hkv, _ = k.shape
    qf, kf, vf = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    out = np.zeros((H, D), np.float32)
    lib.ref_cpu_decode_attn(_ptr(qf, _f32p), _ptr(kf, _f32p), _ptr(vf, _f32p), _ptr(out, _f32p),
                            H, Hkv, D, T)
    return out


# ------------------------------------------------------------ comparisons
def max_errors(x: np.ndarray, ref: np.ndarray, eps: float = 1e-3):
    """(max |x - r|, max |x - r| / max(|r|, eps)) in float64."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(x - ref)
    return float(err.max(initial=0.0)), float((err / np.maximum(np.abs(ref), eps)).max(initial=0.0))
