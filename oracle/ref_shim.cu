// ref_shim.cu - C entry points into the reference's own code, for parity checks.
//
// TEST INFRASTRUCTURE ONLY (see decode_attn_oracle.c).  The Makefile in this
// directory compiles this shim together with the reference's unmodified
// sources, read in place from the reference tree, into oracle/_ref/:
//   * tests/test_kernels.cpp is included whole (its main() renamed) so its
//     static CPU oracle cpu_decode_attn (:229-270) becomes callable;
//   * kernels/*.cu are compiled for sm_100a with the reference's own flags
//     (-O3 --use_fast_math, CMakeLists.txt:38-44), giving the reference GPU
//     kernels decode_attn_v4_flash and prefill_attn_causal.
// Nothing here is shipped; the product library never links it.
#define main forgert_reference_test_main
#include "test_kernels.cpp"
#undef main

#include <thread>
#include <vector>

extern "C" {

// The reference CPU oracle, tests/test_kernels.cpp:229-270 (fp32 in/out).
void ref_cpu_decode_attn(const float* q, const float* k_cache, const float* v_cache, float* out,
                         int num_heads, int num_kv_heads, int head_dim, int kv_len) {
    std::vector<float> qv(q, q + (size_t)num_heads * head_dim);
    std::vector<float> kv(k_cache, k_cache + (size_t)kv_len * num_kv_heads * head_dim);
    std::vector<float> vv(v_cache, v_cache + (size_t)kv_len * num_kv_heads * head_dim);
    std::vector<float> o = cpu_decode_attn(qv, kv, vv, num_heads, num_kv_heads, head_dim, kv_len);
    std::copy(o.begin(), o.end(), out);
}

// Runs `calls` independent cpu_decode_attn problems on `threads` host threads.
// Problem i reads q_i, k_i, v_i and writes out_i (fp32 arrays, see above).
// This is the CPU baseline arm of the benchmark: the reference's own code,
// spread over the host cores the way a serving process would spread layers.
void ref_cpu_decode_attn_many(const float* const* qs, const float* const* ks,
                              const float* const* vs, float* const* outs, const int* kv_lens,
                              int calls, int num_heads, int num_kv_heads, int head_dim,
                              int threads) {
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    for (int w = 0; w < threads; ++w) {
        pool.emplace_back([=]() {
            for (int i = w; i < calls; i += threads)
                ref_cpu_decode_attn(qs[i], ks[i], vs[i], outs[i], num_heads, num_kv_heads,
                                    head_dim, kv_lens[i]);
        });
    }
    for (auto& t : pool) t.join();
}

// The reference GPU kernels (device pointers, legacy default stream when null).
void ref_decode_attn_v4_flash(const void* q, const void* k, const void* v, void* out,
                              int num_heads, int num_kv_heads, int head_dim, int kv_len,
                              void* stream) {
    decode_attn_v4_flash(static_cast<const __half*>(q), static_cast<const __half*>(k),
                         static_cast<const __half*>(v), static_cast<__half*>(out), num_heads,
                         num_kv_heads, head_dim, kv_len, static_cast<cudaStream_t>(stream));
}

void ref_prefill_attn_causal(const void* q, const void* k, const void* v, void* out, int seq_len,
                             int num_heads, int num_kv_heads, int head_dim, void* stream) {
    prefill_attn_causal(static_cast<const __half*>(q), static_cast<const __half*>(k),
                        static_cast<const __half*>(v), static_cast<__half*>(out), seq_len,
                        num_heads, num_kv_heads, head_dim, static_cast<cudaStream_t>(stream));
}

void ref_rope_v2_fused(void* q, void* k, const float* cos_tab, const float* sin_tab, int seq_len,
                       int num_q_heads, int num_kv_heads, int head_dim, int pos_offset,
                       void* stream) {
    rope_v2_fused(static_cast<__half*>(q), static_cast<__half*>(k), cos_tab, sin_tab, seq_len,
                  num_q_heads, num_kv_heads, head_dim, pos_offset, static_cast<cudaStream_t>(stream));
}

// The reference's RoPE tables (kernels/rope.cu:28-56: its own allocation and
// kernel), copied into caller-owned device buffers.
int ref_rope_precompute_tables(float* cos_out, float* sin_out, int max_seq_len, int head_dim,
                               float base, float scale) {
    float* c = nullptr;
    float* s = nullptr;
    rope_precompute_tables(&c, &s, max_seq_len, head_dim, base, scale);
    const size_t bytes = (size_t)max_seq_len * (head_dim / 2) * sizeof(float);
    cudaError_t e = cudaMemcpy(cos_out, c, bytes, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(sin_out, s, bytes, cudaMemcpyDeviceToDevice);
    cudaFree(c);
    cudaFree(s);
    return (int)e;
}

void ref_bias_add_broadcast(void* out, const void* bias, int seq_len, int hidden, void* stream) {
    bias_add_broadcast(static_cast<__half*>(out), static_cast<const __half*>(bias), seq_len,
                       hidden, static_cast<cudaStream_t>(stream));
}

// The reference's own kernel test program (14 checks); returns its exit code.
int ref_run_kernel_tests(void) { return forgert_reference_test_main(); }

}  // extern "C"
