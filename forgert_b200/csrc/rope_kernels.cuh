// rope_kernels.cuh - fused decode prologue: RoPE on q/k + KV-cache append.
//
// Replaces, per layer and step, the reference sequence
//   rope_v2_fused(q, k, ...)                      kernels/rope.cu:162-207
//   cudaMemcpyAsync(k_cache + pos*Hkv*D, k, ...)  runtime/executor.cpp:145-148
//   cudaMemcpyAsync(v_cache + pos*Hkv*D, v, ...)  runtime/executor.cpp:149-152
// with one launch.  Rotation convention is the reference's NeoX half split:
// for f < D/2 the pair (x[f], x[f + D/2]) becomes
//   (a*c - b*s, a*s + b*c),  c = cos_tab[pos][f], s = sin_tab[pos][f],
// computed in fp32 and rounded to fp16 once (rope.cu:181-189).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace fr {

// grid = seq_len (one CTA per token), block = 128.
__global__ void rope_append_kernel(__half* __restrict__ q, __half* __restrict__ k,
                                   const __half* __restrict__ v, __half* __restrict__ k_cache,
                                   __half* __restrict__ v_cache, const float* __restrict__ cos_tab,
                                   const float* __restrict__ sin_tab, int num_heads,
                                   int num_kv_heads, int head_dim, int pos_offset) {
    const int tok = blockIdx.x;
    const int pos = tok + pos_offset;
    const int half_d = head_dim >> 1;
    const float* ct = cos_tab + (size_t)pos * half_d;
    const float* st = sin_tab + (size_t)pos * half_d;

    // q heads then k heads: one (head, f) pair per iteration.
    const int qpairs = num_heads * half_d;
    const int kpairs = num_kv_heads * half_d;
    __half* qtok = q + (size_t)tok * num_heads * head_dim;
    __half* ktok = k + (size_t)tok * num_kv_heads * head_dim;
    __half* kdst = k_cache + (size_t)pos * num_kv_heads * head_dim;
    for (int i = threadIdx.x; i < qpairs + kpairs; i += blockDim.x) {
        const bool is_k = i >= qpairs;
        const int j = is_k ? i - qpairs : i;
        const int head = j / half_d;
        const int f = j - head * half_d;
        __half* x = (is_k ? ktok : qtok) + (size_t)head * head_dim;
        const float c = ct[f], s = st[f];
        const float a = __half2float(x[f]);
        const float bb = __half2float(x[f + half_d]);
        const __half r0 = __float2half(a * c - bb * s);
        const __half r1 = __float2half(a * s + bb * c);
        x[f] = r0;
        x[f + half_d] = r1;
        if (is_k) {
            kdst[(size_t)head * head_dim + f] = r0;
            kdst[(size_t)head * head_dim + f + half_d] = r1;
        }
    }
    // v rows: straight copy (16-byte vectors; head_dim*num_kv_heads*2 is a multiple of 16).
    const int vvec = num_kv_heads * head_dim / 8;
    const uint4* vsrc = reinterpret_cast<const uint4*>(v + (size_t)tok * num_kv_heads * head_dim);
    uint4* vdst = reinterpret_cast<uint4*>(v_cache + (size_t)pos * num_kv_heads * head_dim);
    for (int i = threadIdx.x; i < vvec; i += blockDim.x) vdst[i] = vsrc[i];
}

}  // namespace fr
