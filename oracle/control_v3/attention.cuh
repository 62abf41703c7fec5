#pragma once
// control_v3/attention.cuh - TEST INFRASTRUCTURE ONLY (oracle/Makefile,
// engine e2e_v3 of tests/test_e2e_gpu.py).
//
// A control for the end-to-end argmax comparison: the reference runtime
// with the reference's own decode_attn_v3_vec (kernels/attention_decode.cu:
// 309-390) where runtime/executor.cpp calls decode_attn_v4_flash.  Both
// kernels compute the same attention with a different reduction order, so
// this engine shows how far the reference's own argmax moves when only the
// attention kernel's rounding changes.  The declarations below repeat the
// reference's launcher signatures (kernels/attention.cuh:52-82), which the
// reference's attention_decode.cu defines; this header only redirects v4.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

void decode_attn_v3_vec(const __half* __restrict__ q, const __half* __restrict__ k_cache,
                        const __half* __restrict__ v_cache, __half* __restrict__ out,
                        int num_heads, int num_kv_heads, int head_dim, int kv_len,
                        cudaStream_t stream = nullptr);

void prefill_attn_causal(const __half* __restrict__ q, const __half* __restrict__ k,
                         const __half* __restrict__ v, __half* __restrict__ out, int seq_len,
                         int num_heads, int num_kv_heads, int head_dim,
                         cudaStream_t stream = nullptr);

inline void decode_attn_v4_flash(const __half* __restrict__ q, const __half* __restrict__ k_cache,
                                 const __half* __restrict__ v_cache, __half* __restrict__ out,
                                 int num_heads, int num_kv_heads, int head_dim, int kv_len,
                                 cudaStream_t stream = nullptr) {
    decode_attn_v3_vec(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim, kv_len,
                       stream);
}
