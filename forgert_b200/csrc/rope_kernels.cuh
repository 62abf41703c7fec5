// rope_kernels.cuh - fused decode prologue: q/k/v bias add + RoPE on q/k +
// KV-cache append.
//
// Replaces, per layer and step, the reference sequence
//   bias_add_broadcast(q|k|v, bias, ...)  x3      runtime/executor.cpp:135-137,
//                                                 kernels/elementwise.cu:81-98
//   rope_v2_fused(q, k, ...)                      kernels/rope.cu:162-207
//   cudaMemcpyAsync(k_cache + pos*Hkv*D, k, ...)  runtime/executor.cpp:145-148
//   cudaMemcpyAsync(v_cache + pos*Hkv*D, v, ...)  runtime/executor.cpp:149-152
// with one launch.  The bias add is one fp16 addition rounded to nearest
// (__hadd, as elementwise.cu:90); a null bias skips it.  Rotation convention
// is the reference's NeoX half split: for f < D/2 the pair (x[f], x[f + D/2])
// becomes
//   (a*c - b*s, a*s + b*c),  c = cos_tab[pos][f], s = sin_tab[pos][f],
// computed in fp32 and rounded to fp16 once (rope.cu:181-189).  q and k are
// left rotated in place and v biased in place, as the reference sequence
// leaves them.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace fr {

constexpr int kRopeThreads = 256;

// Work items of one token: (H + Hkv) * D/2 rotation pairs, then Hkv * D / 8
// sixteen-byte v vectors; one item per thread.
__host__ __device__ inline int rope_items(int num_heads, int num_kv_heads, int head_dim) {
    return (num_heads + num_kv_heads) * (head_dim / 2) + num_kv_heads * head_dim / 8;
}

// grid = (seq_len, ceil(rope_items / kRopeThreads)), block = kRopeThreads.
__global__ void __launch_bounds__(kRopeThreads)
rope_append_kernel(__half* __restrict__ q, __half* __restrict__ k, __half* __restrict__ v,
                   const __half* __restrict__ q_bias, const __half* __restrict__ k_bias,
                   const __half* __restrict__ v_bias, __half* __restrict__ k_cache,
                   __half* __restrict__ v_cache, const float* __restrict__ cos_tab,
                   const float* __restrict__ sin_tab, int num_heads, int num_kv_heads,
                   int head_dim, int pos_offset) {
    const int tok = blockIdx.x;
    const int pos = tok + pos_offset;
    const int half_d = head_dim >> 1;
    const int qpairs = num_heads * half_d;
    const int kpairs = num_kv_heads * half_d;
    const int i = blockIdx.y * kRopeThreads + threadIdx.x;
    if (i < qpairs + kpairs) {
        // one (head, f) rotation pair of q (first) or k
        const bool is_k = i >= qpairs;
        const int j = is_k ? i - qpairs : i;
        const int head = j / half_d;
        const int f = j - head * half_d;
        const size_t e0 = (size_t)head * head_dim + f;
        __half* x = is_k ? k + (size_t)tok * num_kv_heads * head_dim
                         : q + (size_t)tok * num_heads * head_dim;
        const __half* bias = is_k ? k_bias : q_bias;
        __half x0 = x[e0], x1 = x[e0 + half_d];
        if (bias) {
            x0 = __hadd(x0, bias[e0]);
            x1 = __hadd(x1, bias[e0 + half_d]);
        }
        const float c = cos_tab[(size_t)pos * half_d + f];
        const float s = sin_tab[(size_t)pos * half_d + f];
        const float a = __half2float(x0);
        const float bb = __half2float(x1);
        const __half r0 = __float2half(a * c - bb * s);
        const __half r1 = __float2half(a * s + bb * c);
        x[e0] = r0;
        x[e0 + half_d] = r1;
        if (is_k) {
            __half* kdst = k_cache + (size_t)pos * num_kv_heads * head_dim;
            kdst[e0] = r0;
            kdst[e0 + half_d] = r1;
        }
        return;
    }
    // one 16-byte vector of the v row (head_dim*num_kv_heads*2 is a multiple
    // of 16), biased first when a bias is given
    const int vi = i - qpairs - kpairs;
    if (vi >= num_kv_heads * head_dim / 8) return;
    uint4* vsrc = reinterpret_cast<uint4*>(v + (size_t)tok * num_kv_heads * head_dim);
    uint4* vdst = reinterpret_cast<uint4*>(v_cache + (size_t)pos * num_kv_heads * head_dim);
    uint4 xv = vsrc[vi];
    if (v_bias) {
        const uint4 bv = reinterpret_cast<const uint4*>(v_bias)[vi];
        __half2* xh = reinterpret_cast<__half2*>(&xv);
        const __half2* bh = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
        for (int u = 0; u < 4; ++u) xh[u] = __hadd2(xh[u], bh[u]);
        vsrc[vi] = xv;
    }
    vdst[vi] = xv;
}

// RoPE tables on the device with the reference's single-precision
// arithmetic.  The reference builds them with
//   theta = pos / (powf(base, 2 * f / head_dim) * scale), cosf, sinf
// (kernels/rope.cu:28-42) compiled with --use_fast_math, which turns the
// two divisions, powf, cosf and sinf into the fast approximate intrinsics;
// calling those intrinsics here gives the same table values (the fast
// sine/cosine lose accuracy as theta grows, which the tables then share).
// One thread per (pos, f); grid covers max_seq_len * head_dim / 2 entries.
__global__ void rope_tables_kernel(float* __restrict__ cos_tab, float* __restrict__ sin_tab,
                                   int max_seq_len, int head_dim, float base, float scale) {
    const int half_d = head_dim >> 1;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)max_seq_len * half_d) return;
    const int pos = (int)(i / half_d);
    const int f = (int)(i - (long long)pos * half_d);
    const float expo = __fdividef(2.0f * (float)f, (float)head_dim);
    const float theta = __fdividef((float)pos, __powf(base, expo) * scale);
    cos_tab[i] = __cosf(theta);
    sin_tab[i] = __sinf(theta);
}

}  // namespace fr
