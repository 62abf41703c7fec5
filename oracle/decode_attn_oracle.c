/*
 * decode_attn_oracle.c - CPU restatement of ForgeRT's decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * engine in forgert_b200/: only tests/, __graft_entry__.smoke() and the CPU
 * baseline leg of bench.py may load it.  Nothing in the product links it.
 *
 * Parity is pinned: oracle_decode_attn_f32 is checked bit for bit against
 * the reference's own CPU implementation (cpu_decode_attn, compiled from the
 * reference sources into oracle/_ref) and against committed golden vectors
 * produced from it (tests/golden/).
 *
 * Functions and the reference code they restate:
 *   oracle_decode_attn_f32   cpu_decode_attn, tests/test_kernels.cpp:229-270
 *                            (fp32, two-pass softmax, w = e/denom, o += w*v,
 *                            kv head = h / (H/Hkv)); same operation order.
 *   oracle_decode_attn_f64   the same algorithm in fp64: the exact answer the
 *                            fp16 outputs are compared with.
 *   oracle_decode_attn_batched_f64
 *                            one f64 decode per sequence (the reference has no
 *                            batch; it is B independent decode_attn_v4_flash
 *                            calls, kernels/attention.cuh:65-71).
 *   oracle_partial_f64 / oracle_merge_f64
 *                            split-KV (m, l, acc) states in base 2 and their
 *                            log-sum-exp merge (flash-decoding algebra).
 *   oracle_prefill_f64       prefill_attn_kernel, kernels/attention_decode.cu:563-609
 *                            (causal: position s attends to 0..s).
 *   oracle_rope_tables_f64   compute_rope_tables_kernel, kernels/rope.cu:28-42,
 *                            theta = pos / (base^(2f/D) * scale), in fp64.
 *   oracle_rope_append       rope_kernel_v2_fused, kernels/rope.cu:162-191, plus
 *                            the KV append of runtime/executor.cpp:145-152.
 *   oracle_qkv_bias_rope_append
 *                            the same preceded by the q/k/v bias adds of
 *                            runtime/executor.cpp:135-137 (bias_broadcast_kernel,
 *                            kernels/elementwise.cu:81-91).
 *
 * fp16 data is passed as raw binary16 bit patterns (uint16_t).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ----------------------------------------------------------- binary16 */
float oracle_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1f;
    const uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: value = man * 2^-24 */
            float f = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* Round-to-nearest-even conversion from double (the exact oracle values). */
uint16_t oracle_double_to_half(double x) {
    uint16_t sign = signbit(x) ? 0x8000 : 0;
    double a = fabs(x);
    if (isnan(x)) return 0x7e00;
    if (a >= 65520.0) return sign | 0x7c00; /* rounds to inf */
    if (a < 6.103515625e-05) {             /* subnormal range: units of 2^-24 */
        double q = a / 5.9604644775390625e-08;
        double r = nearbyint(q);           /* default rounding mode: to nearest even */
        return sign | (uint16_t)r;         /* r == 1024 becomes the smallest normal */
    }
    int e;
    double m = frexp(a, &e);               /* a = m * 2^e, m in [0.5, 1) */
    double q = ldexp(m, 11);               /* 11 significant bits in [1024, 2048) */
    double r = nearbyint(q);
    if (r >= 2048.0) { r = 1024.0; e += 1; }
    int hexp = e - 1 + 15;                 /* a = (r/1024) * 2^(e-1) */
    if (hexp >= 31) return sign | 0x7c00;
    return sign | (uint16_t)(hexp << 10) | (uint16_t)((int)r - 1024);
}

static float h2f(uint16_t h) { return oracle_half_to_float(h); }

/* ------------------------------------------------- cpu_decode_attn (fp32) */
void oracle_decode_attn_f32(const float* q, const float* k_cache, const float* v_cache,
                            float* out, int num_heads, int num_kv_heads, int head_dim,
                            int kv_len) {
    const int gqa = num_heads / num_kv_heads;
    const float scale = 1.f / sqrtf((float)head_dim);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(kv_len > 0 ? kv_len : 1));
    memset(out, 0, sizeof(float) * (size_t)num_heads * head_dim);
    for (int h = 0; h < num_heads; h++) {
        const int kv_h = h / gqa;
        const float* q_h = q + (size_t)h * head_dim;
        float max_s = -1e30f;
        for (int t = 0; t < kv_len; t++) {
            const float* k_t = k_cache + ((size_t)t * num_kv_heads + kv_h) * head_dim;
            float dot = 0.f;
            for (int d = 0; d < head_dim; d++) dot += q_h[d] * k_t[d];
            scores[t] = dot * scale;
            if (max_s < scores[t]) max_s = scores[t];
        }
        float denom = 0.f;
        for (int t = 0; t < kv_len; t++) {
            scores[t] = expf(scores[t] - max_s);
            denom += scores[t];
        }
        float* o = out + (size_t)h * head_dim;
        for (int t = 0; t < kv_len; t++) {
            const float* v_t = v_cache + ((size_t)t * num_kv_heads + kv_h) * head_dim;
            const float w = scores[t] / denom;
            for (int d = 0; d < head_dim; d++) o[d] += w * v_t[d];
        }
    }
    free(scores);
}

/* --------------------------------------------------- exact (fp64) decode */
/* q: [H, D], k/v: rows at `row_stride` elements per position, kv head kvh at
 * offset kvh*D.  out: [H, D] fp64. */
static void decode_one_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                           long long row_stride, double* out, int num_heads, int num_kv_heads,
                           int head_dim, int kv_len) {
    const int gqa = num_heads / num_kv_heads;
    const double scale = 1.0 / sqrt((double)head_dim);
    double* scores = (double*)malloc(sizeof(double) * (size_t)(kv_len > 0 ? kv_len : 1));
    for (int h = 0; h < num_heads; h++) {
        const int kv_h = h / gqa;
        double qh[512];
        for (int d = 0; d < head_dim; d++) qh[d] = h2f(q[(size_t)h * head_dim + d]);
        double mx = -INFINITY;
        for (int t = 0; t < kv_len; t++) {
            const uint16_t* kt = k + (size_t)t * row_stride + (size_t)kv_h * head_dim;
            double dot = 0.0;
            for (int d = 0; d < head_dim; d++) dot += qh[d] * (double)h2f(kt[d]);
            scores[t] = dot * scale;
            if (scores[t] > mx) mx = scores[t];
        }
        double denom = 0.0;
        for (int t = 0; t < kv_len; t++) {
            scores[t] = exp(scores[t] - mx);
            denom += scores[t];
        }
        double* o = out + (size_t)h * head_dim;
        for (int d = 0; d < head_dim; d++) o[d] = 0.0;
        for (int t = 0; t < kv_len; t++) {
            const uint16_t* vt = v + (size_t)t * row_stride + (size_t)kv_h * head_dim;
            for (int d = 0; d < head_dim; d++) o[d] += scores[t] * (double)h2f(vt[d]);
        }
        for (int d = 0; d < head_dim; d++) o[d] = kv_len > 0 ? o[d] / denom : 0.0;
    }
    free(scores);
}

void oracle_decode_attn_f64(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            double* out, int num_heads, int num_kv_heads, int head_dim,
                            int kv_len) {
    decode_one_f64(q, k_cache, v_cache, (long long)num_kv_heads * head_dim, out, num_heads,
                   num_kv_heads, head_dim, kv_len);
}

/* Sequence b: q + b*H*D, cache rows from caches[b], length kv_lens[b]. */
void oracle_decode_attn_batched_f64(const uint16_t* q, const uint16_t* const* k_caches,
                                    const uint16_t* const* v_caches, const int* kv_lens,
                                    double* out, int batch, int num_heads, int num_kv_heads,
                                    int head_dim) {
    for (int b = 0; b < batch; b++)
        decode_one_f64(q + (size_t)b * num_heads * head_dim, k_caches[b], v_caches[b],
                       (long long)num_kv_heads * head_dim,
                       out + (size_t)b * num_heads * head_dim, num_heads, num_kv_heads,
                       head_dim, kv_lens[b]);
}

/* Partial state over positions [begin, end): m = max_t s_t*log2(e)/sqrt(D)
 * (the base-2 score), l = sum_t 2^(s2_t - m), acc[d] = sum_t 2^(s2_t - m) v_t[d].
 * Empty range: m = -inf, l = 0, acc = 0. */
void oracle_partial_f64(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                        int begin, int end, double* m_out, double* l_out, double* acc_out,
                        int num_heads, int num_kv_heads, int head_dim) {
    const int gqa = num_heads / num_kv_heads;
    const long long rs = (long long)num_kv_heads * head_dim;
    const double sl2 = 1.4426950408889634 / sqrt((double)head_dim);
    const int n = end > begin ? end - begin : 0;
    double* s2 = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    for (int h = 0; h < num_heads; h++) {
        const int kv_h = h / gqa;
        double mx = -INFINITY;
        for (int i = 0; i < n; i++) {
            const uint16_t* kt = k_cache + (size_t)(begin + i) * rs + (size_t)kv_h * head_dim;
            double dot = 0.0;
            for (int d = 0; d < head_dim; d++)
                dot += (double)h2f(q[(size_t)h * head_dim + d]) * (double)h2f(kt[d]);
            s2[i] = dot * sl2;
            if (s2[i] > mx) mx = s2[i];
        }
        double l = 0.0;
        double* acc = acc_out + (size_t)h * head_dim;
        for (int d = 0; d < head_dim; d++) acc[d] = 0.0;
        for (int i = 0; i < n; i++) {
            const double w = exp2(s2[i] - mx);
            l += w;
            const uint16_t* vt = v_cache + (size_t)(begin + i) * rs + (size_t)kv_h * head_dim;
            for (int d = 0; d < head_dim; d++) acc[d] += w * (double)h2f(vt[d]);
        }
        m_out[h] = mx;
        l_out[h] = l;
    }
    free(s2);
}

/* Merge of num_states states per head, stacked state-major ([S, H] / [S, H, D]). */
void oracle_merge_f64(const double* m, const double* l, const double* acc, int num_states,
                      double* out, int num_heads, int head_dim) {
    for (int h = 0; h < num_heads; h++) {
        double mx = -INFINITY;
        for (int s = 0; s < num_states; s++)
            if (m[(size_t)s * num_heads + h] > mx) mx = m[(size_t)s * num_heads + h];
        const double mu = isinf(mx) ? 0.0 : mx;
        double lt = 0.0;
        for (int d = 0; d < head_dim; d++) out[(size_t)h * head_dim + d] = 0.0;
        for (int s = 0; s < num_states; s++) {
            const size_t i = (size_t)s * num_heads + h;
            const double w = exp2(m[i] - mu);
            lt += l[i] * w;
            for (int d = 0; d < head_dim; d++)
                out[(size_t)h * head_dim + d] += acc[i * head_dim + d] * w;
        }
        for (int d = 0; d < head_dim; d++)
            out[(size_t)h * head_dim + d] = lt > 0.0 ? out[(size_t)h * head_dim + d] / lt : 0.0;
    }
}

/* Causal prefill: q [T, H, D], k/v [T, Hkv, D]; out [T, H, D] fp64. */
void oracle_prefill_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v, double* out,
                        int seq_len, int num_heads, int num_kv_heads, int head_dim) {
    for (int s = 0; s < seq_len; s++)
        decode_one_f64(q + (size_t)s * num_heads * head_dim, k, v,
                       (long long)num_kv_heads * head_dim,
                       out + (size_t)s * num_heads * head_dim, num_heads, num_kv_heads,
                       head_dim, s + 1);
}

/* RoPE tables [max_seq_len, D/2], fp64 evaluation rounded to fp32. */
void oracle_rope_tables_f64(float* cos_tab, float* sin_tab, int max_seq_len, int head_dim,
                            double base, double scale) {
    const int half_d = head_dim / 2;
    for (int pos = 0; pos < max_seq_len; pos++)
        for (int f = 0; f < half_d; f++) {
            const double th = (double)pos / (pow(base, 2.0 * f / (double)head_dim) * scale);
            cos_tab[(size_t)pos * half_d + f] = (float)cos(th);
            sin_tab[(size_t)pos * half_d + f] = (float)sin(th);
        }
}

/* In-place NeoX rotation of x [T, heads, D] at positions pos_offset + t,
 * fp32 math, one fp16 rounding per output (rope.cu:180-190). */
static void rope_inplace(uint16_t* x, const float* cos_tab, const float* sin_tab, int seq_len,
                         int heads, int head_dim, int pos_offset) {
    const int half_d = head_dim / 2;
    for (int t = 0; t < seq_len; t++)
        for (int h = 0; h < heads; h++) {
            uint16_t* row = x + ((size_t)t * heads + h) * head_dim;
            const int pos = t + pos_offset;
            for (int f = 0; f < half_d; f++) {
                const float c = cos_tab[(size_t)pos * half_d + f];
                const float s = sin_tab[(size_t)pos * half_d + f];
                const float a = h2f(row[f]);
                const float b = h2f(row[f + half_d]);
                const float r0 = a * c - b * s;
                const float r1 = a * s + b * c;
                row[f] = oracle_double_to_half((double)r0);
                row[f + half_d] = oracle_double_to_half((double)r1);
            }
        }
}

/* x[t, :] += bias[:] in fp16: the exact sum rounded once to nearest-even,
 * which is what __hadd computes (bias_broadcast_kernel,
 * kernels/elementwise.cu:81-91).  A NULL bias leaves x unchanged. */
static void bias_add_f16(uint16_t* x, const uint16_t* bias, int rows, int width) {
    if (!bias) return;
    for (int t = 0; t < rows; t++)
        for (int d = 0; d < width; d++) {
            uint16_t* e = x + (size_t)t * width + d;
            *e = oracle_double_to_half((double)h2f(*e) + (double)h2f(bias[d]));
        }
}

/* The reference's decode prologue with projection biases
 * (runtime/executor.cpp:135-152): q/k/v += bias, RoPE on q and k, then the
 * k/v rows appended to the cache at pos_offset + t.  q, k, v are updated in
 * place like the reference's activation buffers. */
void oracle_qkv_bias_rope_append(uint16_t* q, uint16_t* k, uint16_t* v, const uint16_t* q_bias,
                                 const uint16_t* k_bias, const uint16_t* v_bias,
                                 uint16_t* k_cache, uint16_t* v_cache, const float* cos_tab,
                                 const float* sin_tab, int seq_len, int num_heads,
                                 int num_kv_heads, int head_dim, int pos_offset) {
    bias_add_f16(q, q_bias, seq_len, num_heads * head_dim);
    bias_add_f16(k, k_bias, seq_len, num_kv_heads * head_dim);
    bias_add_f16(v, v_bias, seq_len, num_kv_heads * head_dim);
    rope_inplace(q, cos_tab, sin_tab, seq_len, num_heads, head_dim, pos_offset);
    rope_inplace(k, cos_tab, sin_tab, seq_len, num_kv_heads, head_dim, pos_offset);
    const size_t row = (size_t)num_kv_heads * head_dim;
    memcpy(k_cache + (size_t)pos_offset * row, k, sizeof(uint16_t) * row * seq_len);
    memcpy(v_cache + (size_t)pos_offset * row, v, sizeof(uint16_t) * row * seq_len);
}

/* RoPE on q and k in place, then k/v rows appended to the cache at
 * pos_offset + t (cache rows have num_kv_heads*D elements). */
void oracle_rope_append(uint16_t* q, uint16_t* k, const uint16_t* v, uint16_t* k_cache,
                        uint16_t* v_cache, const float* cos_tab, const float* sin_tab,
                        int seq_len, int num_heads, int num_kv_heads, int head_dim,
                        int pos_offset) {
    rope_inplace(q, cos_tab, sin_tab, seq_len, num_heads, head_dim, pos_offset);
    rope_inplace(k, cos_tab, sin_tab, seq_len, num_kv_heads, head_dim, pos_offset);
    const size_t row = (size_t)num_kv_heads * head_dim;
    memcpy(k_cache + (size_t)pos_offset * row, k, sizeof(uint16_t) * row * seq_len);
    memcpy(v_cache + (size_t)pos_offset * row, v, sizeof(uint16_t) * row * seq_len);
}
