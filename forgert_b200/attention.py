"""Python mirror of ForgeRT's attention launcher interface (kernels/attention.cuh).

Same names, argument order and meaning as the reference's C++ launchers;
every call goes straight to libforgert_b200.so through the C ABI of
include/forgert_attn.h.  Arguments that are device buffers accept either a
CUDA torch tensor or a raw device pointer (int); `stream` is a
torch.cuda.Stream, a raw cudaStream_t (int) or None (the legacy default
stream, as in the reference).  Errors raise ForgeRTError, as the reference's
CUDA_CHECK raises std::runtime_error.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

from ._lib import ForgeRTError, check, load

__all__ = [
    "ForgeRTError", "decode_attn_v4_flash", "decode_attn_v0_naive", "decode_attn_v1_coal",
    "decode_attn_v2_warp_red", "decode_attn_v3_vec", "prefill_attn_causal",
    "decode_attn_batched", "decode_attn_partial", "lse_merge", "rope_precompute_tables",
    "rope_tables_device",
    "rope_append", "reserve_workspace", "decode_workspace_size", "device_error",
]


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    dp = getattr(x, "data_ptr", None)
    if dp is None:
        raise TypeError(f"expected a device tensor or pointer, got {type(x).__name__}")
    if not getattr(x, "is_cuda", True):
        raise ValueError("tensor must live on a CUDA device")
    return dp()


def _stream(s) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return getattr(s, "cuda_stream", None) or getattr(s, "stream_id", None) or s


def decode_attn_v4_flash(q, k_cache, v_cache, out, num_heads: int, num_kv_heads: int,
                         head_dim: int, kv_len: int, stream=None) -> None:
    """Decode attention for one token (kernels/attention.cuh:65-71).

    q/out [num_heads, head_dim] fp16; k_cache/v_cache one layer's
    [>= kv_len, num_kv_heads, head_dim] fp16 view of the cache.
    """
    lib = load()
    check("fr_decode_attn", lib.fr_decode_attn(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), num_heads, num_kv_heads, head_dim,
        kv_len, _stream(stream)))


# The reference keeps its earlier versions under their own names
# (attention.cuh:29-62); they compute the same function, so they all reach
# the one B200 kernel.
decode_attn_v0_naive = decode_attn_v4_flash
decode_attn_v1_coal = decode_attn_v4_flash
decode_attn_v2_warp_red = decode_attn_v4_flash
decode_attn_v3_vec = decode_attn_v4_flash


def prefill_attn_causal(q, k, v, out, seq_len: int, num_heads: int, num_kv_heads: int,
                        head_dim: int, stream=None) -> None:
    """Causal prefill (kernels/attention.cuh:76-82): q/out [seq_len, H, D],
    k/v [seq_len, Hkv, D]."""
    lib = load()
    check("fr_prefill_attn", lib.fr_prefill_attn(
        _ptr(q), _ptr(k), _ptr(v), _ptr(out), seq_len, num_heads, num_kv_heads, head_dim,
        _stream(stream)))


def decode_attn_batched(q, k_pool, v_pool, row_offsets, kv_lens, out, batch: int,
                        num_heads: int, num_kv_heads: int, head_dim: int, pool_rows: int,
                        max_kv_len: int, stream=None) -> None:
    """Ragged batch over a KV pool [pool_rows, Hkv, D]: sequence b's rows start
    at row_offsets[b] (device int64) and it has kv_lens[b] (device int32) of them."""
    lib = load()
    check("fr_decode_attn_batched", lib.fr_decode_attn_batched(
        _ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(row_offsets), _ptr(kv_lens), _ptr(out), batch,
        num_heads, num_kv_heads, head_dim, pool_rows, max_kv_len, _stream(stream)))


def decode_attn_paged(q, k_pages, v_pages, block_table, kv_lens, out, batch: int,
                      num_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                      num_pages: int, max_blocks_per_seq: int, max_kv_len: int,
                      stream=None) -> None:
    """Batch over a paged cache [num_pages, page_size, Hkv, D]: position t of
    sequence b is row t % page_size of page block_table[b, t // page_size]
    (device int32 [batch, max_blocks_per_seq]); kv_lens device int32."""
    lib = load()
    check("fr_decode_attn_paged", lib.fr_decode_attn_paged(
        _ptr(q), _ptr(k_pages), _ptr(v_pages), _ptr(block_table), _ptr(kv_lens), _ptr(out),
        batch, num_heads, num_kv_heads, head_dim, page_size, num_pages, max_blocks_per_seq,
        max_kv_len, _stream(stream)))


def decode_attn_partial(q, k_cache, v_cache, kv_len: int, state_ml, state_acc, num_heads: int,
                        num_kv_heads: int, head_dim: int, stream=None) -> None:
    """(m, l, acc) log-sum-exp state per head over positions [0, kv_len)."""
    lib = load()
    check("fr_decode_attn_partial", lib.fr_decode_attn_partial(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), kv_len, _ptr(state_ml), _ptr(state_acc),
        num_heads, num_kv_heads, head_dim, _stream(stream)))


def lse_merge(states_ml, states_acc, num_states: int, out, num_heads: int, head_dim: int,
              stream=None) -> None:
    """Merge state-major stacked states ([S, H, 2] and [S, H, D] fp32) to fp16 out [H, D]."""
    lib = load()
    check("fr_lse_merge", lib.fr_lse_merge(
        _ptr(states_ml), _ptr(states_acc), num_states, _ptr(out), num_heads, head_dim,
        _stream(stream)))


def rope_precompute_tables(max_seq_len: int, head_dim: int, base: float, scale: float = 1.0,
                           device=None):
    """cos/sin tables [max_seq_len, head_dim/2] fp32 on the device
    (kernels/rope.cuh:227-231); returns (cos, sin) torch tensors."""
    import torch

    lib = load()
    dev = torch.device("cuda") if device is None else torch.device(device)
    cos = torch.empty((max_seq_len, head_dim // 2), dtype=torch.float32, device=dev)
    sin = torch.empty_like(cos)
    with torch.cuda.device(dev):
        check("fr_rope_tables", lib.fr_rope_tables(
            cos.data_ptr(), sin.data_ptr(), max_seq_len, head_dim, float(base), float(scale)))
    return cos, sin


def rope_tables_device(max_seq_len: int, head_dim: int, base: float, scale: float = 1.0,
                       device=None, stream=None):
    """The reference's own table values (fast single-precision arithmetic,
    kernels/rope.cu:28-42), computed on the device; returns (cos, sin)."""
    import torch

    lib = load()
    dev = torch.device("cuda") if device is None else torch.device(device)
    cos = torch.empty((max_seq_len, head_dim // 2), dtype=torch.float32, device=dev)
    sin = torch.empty_like(cos)
    with torch.cuda.device(dev):
        check("fr_rope_tables_device", lib.fr_rope_tables_device(
            cos.data_ptr(), sin.data_ptr(), max_seq_len, head_dim, float(base), float(scale),
            _stream(stream)))
    return cos, sin


def rope_append(q, k, v, k_cache, v_cache, cos_tab, sin_tab, seq_len: int, num_heads: int,
                num_kv_heads: int, head_dim: int, pos_offset: int, stream=None) -> None:
    """RoPE on q/k in place + KV append at rows pos_offset.. (one launch)."""
    lib = load()
    check("fr_rope_append", lib.fr_rope_append(
        _ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(cos_tab), _ptr(sin_tab),
        seq_len, num_heads, num_kv_heads, head_dim, pos_offset, _stream(stream)))


def qkv_bias_rope_append(q, k, v, q_bias, k_bias, v_bias, k_cache, v_cache, cos_tab, sin_tab,
                         seq_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
                         pos_offset: int, stream=None) -> None:
    """q/k/v += bias (None = no bias), RoPE on q/k, KV append: one launch in
    place of runtime/executor.cpp:135-152's six."""
    lib = load()
    check("fr_qkv_bias_rope_append", lib.fr_qkv_bias_rope_append(
        _ptr(q), _ptr(k), _ptr(v), _ptr(q_bias), _ptr(k_bias), _ptr(v_bias), _ptr(k_cache),
        _ptr(v_cache), _ptr(cos_tab), _ptr(sin_tab), seq_len, num_heads, num_kv_heads, head_dim,
        pos_offset, _stream(stream)))


EXCHANGE_HEADER_BYTES = 256          # u32 epoch, u32 done


def exchange_layout(num_heads: int, head_dim: int, world: int) -> dict:
    """Byte offsets inside one rank's exchange buffer (fr_exchange_bytes):
    header, then ml [2][world][H][2] and acc [2][world][H][D] 8-byte words
    indexed [call parity][source rank]; a word is (call epoch << 32) | fp32
    bits."""
    ml = EXCHANGE_HEADER_BYTES
    acc = ml + 2 * world * num_heads * 2 * 8
    return {"header": 0, "ml": ml, "acc": acc,
            "bytes": acc + 2 * world * num_heads * head_dim * 8}


def decode_attn_exchange(q, k_local, v_local, local_kv_len: int, out, num_heads: int,
                         num_kv_heads: int, head_dim: int, bufs, rank: int, world: int,
                         stream=None) -> None:
    """This GPU's KV range + the in-kernel exchange of states with the other
    ranks (bufs: every rank's exchange buffer as seen from here)."""
    import ctypes

    lib = load()
    arr = (ctypes.c_void_p * world)(*[_ptr(b) for b in bufs])
    check("fr_decode_attn_exchange", lib.fr_decode_attn_exchange(
        _ptr(q), _ptr(k_local) if local_kv_len else None, _ptr(v_local) if local_kv_len else None,
        local_kv_len, _ptr(out), num_heads, num_kv_heads, head_dim, arr, rank, world,
        _stream(stream)))


def copy_async(dst, src, nbytes: int | None = None, stream=None) -> None:
    """fr_copy_async: stream-ordered kernel copy; dst/src are CUDA tensors,
    page-locked host tensors (``pin_memory()``) or raw pointers."""
    def addr(x):
        if isinstance(x, int):
            return x
        if not (x.is_cuda or x.is_pinned()):
            raise ValueError("host tensors must be page-locked (pin_memory())")
        return x.data_ptr()

    if nbytes is None:
        nbytes = min(dst.numel() * dst.element_size(), src.numel() * src.element_size())
    check("fr_copy_async", load().fr_copy_async(addr(dst), addr(src), nbytes, _stream(stream)))


def reserve_workspace(nbytes: int) -> None:
    lib = load()
    check("fr_reserve_workspace", lib.fr_reserve_workspace(nbytes))


def prefill_workspace_size(seq_len: int, num_heads: int, head_dim: int) -> int:
    return int(load().fr_prefill_workspace_size(seq_len, num_heads, head_dim))


def decode_workspace_size(batch: int, num_heads: int, num_kv_heads: int, head_dim: int,
                          max_kv_len: int) -> int:
    return int(load().fr_decode_workspace_size(batch, num_heads, num_kv_heads, head_dim,
                                               max_kv_len))


def device_error(clear: bool = True) -> int:
    """In-kernel error word of the current device (0 = none); synchronises."""
    lib = load()
    code = ctypes.c_int(0)
    lib.fr_get_device_error(1 if clear else 0, ctypes.byref(code))
    return code.value
