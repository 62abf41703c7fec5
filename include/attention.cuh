#pragma once
// ---------------------------------------------------------------------------
// attention.cuh - drop-in replacement for ForgeRT's kernels/attention.cuh.
//
// Same file name, function names, parameter lists and default arguments as
// the reference header (kernels/attention.cuh:29-82), so
// runtime/executor.cpp (which includes "attention.cuh" at executor.cpp:19
// and calls decode_attn_v4_flash / prefill_attn_causal at executor.cpp:158-170)
// compiles unchanged when this directory precedes the reference's kernels/
// directory on the include path, and links against libforgert_b200.so.
//
// The functions are header-only forwards to the C ABI in forgert_attn.h.
// The reference launchers return void and never check their launches; here
// a non-zero status throws std::runtime_error, the same exception type the
// reference's CUDA_CHECK raises (runtime/include/types.h:18-26).
// The five decode versions (v0..v4) of the reference compute the same
// function; all of them reach the one sm_100a kernel.
// ---------------------------------------------------------------------------
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "forgert_attn.h"

namespace forgert_b200_detail {
// The default stream of the including translation unit: a null stream means
// the legacy default stream, or this thread's default stream when the
// caller is compiled with --default-stream per-thread (as a launch
// `<<<g, b, 0, nullptr>>>` in that unit would).
inline void* caller_stream(cudaStream_t stream) {
#ifdef CUDA_API_PER_THREAD_DEFAULT_STREAM
    if (stream == nullptr) return static_cast<void*>(cudaStreamPerThread);
#endif
    return static_cast<void*>(stream);
}
inline void throw_if(int status, const char* fn) {
    if (status != FR_OK)
        throw std::runtime_error(std::string("forgert_b200 ") + fn + ": " +
                                 fr_status_string(status));
}
inline void decode(const __half* q, const __half* k_cache, const __half* v_cache, __half* out,
                   int num_heads, int num_kv_heads, int head_dim, int kv_len,
                   cudaStream_t stream, const char* fn) {
    throw_if(fr_decode_attn(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim, kv_len,
                            caller_stream(stream)),
             fn);
}
}  // namespace forgert_b200_detail

// Decode attention  (seq_len == 1; q [1, num_heads, head_dim],
// k_cache/v_cache [kv_len, num_kv_heads, head_dim], out [1, num_heads, head_dim])

inline void decode_attn_v0_naive(const __half* __restrict__ q, const __half* __restrict__ k_cache,
                                 const __half* __restrict__ v_cache, __half* __restrict__ out,
                                 int num_heads, int num_kv_heads, int head_dim, int kv_len,
                                 cudaStream_t stream = nullptr) {
    forgert_b200_detail::decode(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim,
                                kv_len, stream, "decode_attn_v0_naive");
}

inline void decode_attn_v1_coal(const __half* __restrict__ q, const __half* __restrict__ k_cache,
                                const __half* __restrict__ v_cache, __half* __restrict__ out,
                                int num_heads, int num_kv_heads, int head_dim, int kv_len,
                                cudaStream_t stream = nullptr) {
    forgert_b200_detail::decode(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim,
                                kv_len, stream, "decode_attn_v1_coal");
}

inline void decode_attn_v2_warp_red(const __half* __restrict__ q,
                                    const __half* __restrict__ k_cache,
                                    const __half* __restrict__ v_cache, __half* __restrict__ out,
                                    int num_heads, int num_kv_heads, int head_dim, int kv_len,
                                    cudaStream_t stream = nullptr) {
    forgert_b200_detail::decode(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim,
                                kv_len, stream, "decode_attn_v2_warp_red");
}

inline void decode_attn_v3_vec(const __half* __restrict__ q, const __half* __restrict__ k_cache,
                               const __half* __restrict__ v_cache, __half* __restrict__ out,
                               int num_heads, int num_kv_heads, int head_dim, int kv_len,
                               cudaStream_t stream = nullptr) {
    forgert_b200_detail::decode(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim,
                                kv_len, stream, "decode_attn_v3_vec");
}

inline void decode_attn_v4_flash(const __half* __restrict__ q, const __half* __restrict__ k_cache,
                                 const __half* __restrict__ v_cache, __half* __restrict__ out,
                                 int num_heads, int num_kv_heads, int head_dim, int kv_len,
                                 cudaStream_t stream = nullptr) {
    forgert_b200_detail::decode(q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim,
                                kv_len, stream, "decode_attn_v4_flash");
}

// Prefill causal attention  (q/out [seq_len, num_heads, head_dim],
// k/v [seq_len, num_kv_heads, head_dim]; position s attends to 0..s)
inline void prefill_attn_causal(const __half* __restrict__ q, const __half* __restrict__ k,
                                const __half* __restrict__ v, __half* __restrict__ out,
                                int seq_len, int num_heads, int num_kv_heads, int head_dim,
                                cudaStream_t stream = nullptr) {
    forgert_b200_detail::throw_if(
        fr_prefill_attn(q, k, v, out, seq_len, num_heads, num_kv_heads, head_dim,
                        forgert_b200_detail::caller_stream(stream)),
        "prefill_attn_causal");
}
