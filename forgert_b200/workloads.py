"""Seeded synthetic inputs for the five benchmark configurations.

All values are fp16 drawn i.i.d. N(0, 1) (numpy `default_rng`, then rounded
to fp16), in this draw order:

  cfg1  Qwen2-0.5B one layer: H14 Hkv2 D64 kv512, seed 0: q [14,64], K [512,2,64], V.
  cfg2  Qwen2-1.5B sweep: H12 Hkv2 D128, 28 layers of a [28,2,16384,2,128]
        cache, kv_len in {512, 2048, 4096, 16384}.  Layer l's K then V come
        from default_rng([1, l]); q for layer l from default_rng([1, 1000 + l]).
        (Per-layer streams let a test regenerate one layer without the
        other 27.)  RoPE theta 1e6.
  cfg3  Qwen2-7B batched: B64 H28 Hkv4 D128, seed 2: kv_lens = integers in
        [1024, 8192] (64 draws) first, then q [64,28,128], then K_b, V_b per
        sequence b in order.
  cfg4  Qwen2-7B long context: B1 H28 Hkv4 D128 kv131072, seed 3: q, K, V.
  ref   the reference's own kernel-test shapes (tests/test_kernels.cpp:298-339):
        H8 Hkv2 D64 kv128 (+ kv1, + D128), here U(-0.5, 0.5) from numpy.

Algorithmic bytes per decode call (K+V of the valid range + q + out), the
numerator of every GB/s figure: sum_b 2*kv_len_b*Hkv*D*2 + 2*B*H*D*2.
"""
from __future__ import annotations

import numpy as np

CFG2_LAYERS = 28
CFG2_MAX_SEQ = 16384
CFG2_KV_LENS = (512, 2048, 4096, 16384)
CFG2_SHAPE = dict(H=12, Hkv=2, D=128)
CFG1_SHAPE = dict(H=14, Hkv=2, D=64, kv_len=512)
CFG3_SHAPE = dict(B=64, H=28, Hkv=4, D=128, kv_lo=1024, kv_hi=8192)
CFG4_SHAPE = dict(H=28, Hkv=4, D=128, kv_len=131072)
ROPE_THETA = 1e6


def normal_fp16(rng: np.random.Generator, shape) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32).astype(np.float16)


def decode_inputs(seed, H: int, Hkv: int, D: int, kv_len: int, dist: str = "normal"):
    """q [H, D], K, V [kv_len, Hkv, D] fp16 from one stream, in that order."""
    rng = np.random.default_rng(seed)
    if dist == "normal":
        q = normal_fp16(rng, (H, D))
        k = normal_fp16(rng, (kv_len, Hkv, D))
        v = normal_fp16(rng, (kv_len, Hkv, D))
    elif dist == "uniform":
        q = rng.uniform(-0.5, 0.5, (H, D)).astype(np.float16)
        k = rng.uniform(-0.5, 0.5, (kv_len, Hkv, D)).astype(np.float16)
        v = rng.uniform(-0.5, 0.5, (kv_len, Hkv, D)).astype(np.float16)
    else:
        raise ValueError(dist)
    return q, k, v


def cfg1_inputs():
    s = CFG1_SHAPE
    return decode_inputs(0, s["H"], s["Hkv"], s["D"], s["kv_len"])


def cfg2_layer_kv(layer: int, rows: int = CFG2_MAX_SEQ):
    """K, V [rows, 2, 128] of layer `layer` (the first `rows` cache rows)."""
    rng = np.random.default_rng([1, layer])
    shp = (CFG2_MAX_SEQ, CFG2_SHAPE["Hkv"], CFG2_SHAPE["D"])
    k = normal_fp16(rng, shp)
    v = normal_fp16(rng, shp)
    return k[:rows], v[:rows]


def cfg2_layer_q(layer: int):
    rng = np.random.default_rng([1, 1000 + layer])
    return normal_fp16(rng, (CFG2_SHAPE["H"], CFG2_SHAPE["D"]))


def cfg3_lens(seed: int = 2, batch: int = CFG3_SHAPE["B"]) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(CFG3_SHAPE["kv_lo"], CFG3_SHAPE["kv_hi"] + 1, size=batch).astype(np.int32)


def cfg3_inputs(seed: int = 2, batch: int = CFG3_SHAPE["B"], max_seqs: int | None = None):
    """(kv_lens, q [B,H,D], [K_b], [V_b]); `max_seqs` stops after that many sequences."""
    s = CFG3_SHAPE
    rng = np.random.default_rng(seed)
    lens = rng.integers(s["kv_lo"], s["kv_hi"] + 1, size=batch).astype(np.int32)
    q = normal_fp16(rng, (batch, s["H"], s["D"]))
    ks, vs = [], []
    n = batch if max_seqs is None else min(batch, max_seqs)
    for b in range(n):
        ks.append(normal_fp16(rng, (int(lens[b]), s["Hkv"], s["D"])))
        vs.append(normal_fp16(rng, (int(lens[b]), s["Hkv"], s["D"])))
    return lens, q, ks, vs


def cfg4_inputs(seed: int = 3, kv_len: int = CFG4_SHAPE["kv_len"]):
    s = CFG4_SHAPE
    return decode_inputs(seed, s["H"], s["Hkv"], s["D"], kv_len)


def paginate(ks, vs, page_size: int, seed: int = 7, spare_pages: int = 0, fill=np.nan,
             table_width: int | None = None):
    """Lays per-sequence caches ([n_b, Hkv, D] each) out as a paged cache.

    Returns (k_pages, v_pages [num_pages, page_size, Hkv, D], block_table
    [B, table_width] int32).  Pages are handed out in a seeded random order (a
    fragmented serving cache); `spare_pages` extra pages are never referenced;
    unreferenced pages and the rows of each last page past the sequence's end
    hold `fill`; table entries past a sequence's pages are -1."""
    Hkv, D = ks[0].shape[1], ks[0].shape[2]
    need = [-(-int(k.shape[0]) // page_size) for k in ks]
    width = max(1, max(need)) if table_width is None else table_width
    num_pages = sum(need) + spare_pages
    order = np.random.default_rng(seed).permutation(max(num_pages, 1))[:num_pages]
    k_pages = np.full((max(num_pages, 1), page_size, Hkv, D), fill, np.float16)
    v_pages = np.full_like(k_pages, fill)
    table = np.full((len(ks), width), -1, np.int32)
    nxt = 0
    for b, (k, v) in enumerate(zip(ks, vs)):
        n = int(k.shape[0])
        for j in range(need[b]):
            pg = int(order[nxt])
            nxt += 1
            table[b, j] = pg
            rows = slice(j * page_size, min(n, (j + 1) * page_size))
            cnt = rows.stop - rows.start
            k_pages[pg, :cnt] = k[rows]
            v_pages[pg, :cnt] = v[rows]
    return k_pages, v_pages, table


def decode_bytes(kv_lens, H: int, Hkv: int, D: int) -> int:
    """Algorithmic bytes of one decode call over a batch with these lengths."""
    lens = np.atleast_1d(np.asarray(kv_lens, dtype=np.int64))
    return int(2 * lens.sum() * Hkv * D * 2 + 2 * len(lens) * H * D * 2)


def decode_flops(kv_lens, H: int, D: int) -> int:
    lens = np.atleast_1d(np.asarray(kv_lens, dtype=np.int64))
    return int(4 * H * D * lens.sum())
