// prefill_tc_kernels.cuh - causal prefill attention on the 5th-generation
// tensor cores (tcgen05: MMAs issued by one thread, accumulators in tensor
// memory).
//
// Same contract and result as prefill_kernel (prefill_kernels.cuh, the
// mma.sync form kept as an alternative): prefill_attn_causal
// (kernels/attention.cuh:76-82, kernels/attention_decode.cu:563-619), query
// position s of head h attends to positions 0..s of kv head h / (H / Hkv),
// scale 1/sqrt(D), fp32 softmax and accumulation, one fp16 rounding.
//
// One CTA per (128-row query tile, query head), 192 threads, two CTAs per SM:
//   warps 0-3  softmax: thread r owns query row r of the tile (TMEM lane r);
//   warp 4     producer: TMA loads of the Q tile and of the causal K/V tiles
//              (64 positions x D, 128-byte swizzle) through a STAGES ring;
//   warp 5     allocates tensor memory; its lane 0 issues every tcgen05.mma.
// Tensor memory (256 columns per CTA): S [0, 64), P_hi [64, 96), P_lo
// [96, 128) (two fp16 per column), O [128, 128 + D).
// Per K/V tile j:
//   S_j = Q K_j^T          M=128, N=64, K=D; Q and K K-major from the TMA
//                          tiles (shared-memory descriptors, 128B swizzle);
//   softmax                each thread reads its row of S_j (tcgen05.ld),
//                          masks the causal diagonal and rows past T, and
//                          writes P_j = 2^(s - m_ref) as an fp16 pair
//                          (hi + lo, ~22 significant bits) into tensor
//                          memory (tcgen05.st);
//   O += P_j V_j           M=128, N=D, K=64, A = P from tensor memory, B = V
//                          MN-major straight from the TMA tile; hi and lo
//                          accumulate into the same O.
// m_ref is a per-row reference maximum that moves only when a row maximum
// exceeds it by more than 2^8 (so P <= 256); the warp then rescales its rows
// of O in tensor memory between PV_{j-1} and PV_j.  Any reference maximum
// gives the same O / l.  The tensor pipe runs S_{j+1} as soon as the softmax
// warps have read S_j; with two CTAs per SM one CTA's MMAs overlap the other
// CTA's softmax.  Every wait is bounded: on a timeout the kernel records an
// error, stops issuing, waits for its own MMAs and copies and frees tensor
// memory.
#pragma once
#include "decode_kernels.cuh"
#include "prefill_kernels.cuh"
#include "tc_ptx.cuh"

namespace fr {

template <int D, int STAGES>
struct PrefillTcSmem {
    static constexpr int kRows = 128;
    static constexpr int kTile = 64;
    static constexpr int kSub = D / 64;
    static constexpr int kQSubBytes = kRows * 128;
    static constexpr int kQBytes = kSub * kQSubBytes;
    static constexpr int kKvSubBytes = kTile * 128;
    static constexpr int kKvBytes = kSub * kKvSubBytes;
    static constexpr size_t kQOffset = 0;
    static constexpr size_t kKOffset = kQBytes;
    static constexpr size_t kVOffset = kKOffset + size_t(STAGES) * kKvBytes;
    static constexpr size_t kBarOffset = kVOffset + size_t(STAGES) * kKvBytes;
    // q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full, s_free,
    // p_full, pv_full, done; then the TMEM base address slot
    static constexpr int kNumBars = 1 + 4 * STAGES + 5;
    static constexpr size_t kBytes = 1024 + kBarOffset + kNumBars * sizeof(uint64_t) + 16;
    static constexpr uint32_t kPhiCol = 64, kPloCol = 96, kOCol = 128;
    static constexpr uint32_t kTmemCols = 256;
};

// Reference-maximum slack in log2 units: P = 2^(s - m_ref) <= 2^8.
constexpr float kRescaleLog2 = 8.f;

// Most units one query tile's K/V range is split into.
constexpr int kMaxPrefillChunks = 4;

// 64 outputs of one row, scaled by inv, as fp16 (16-byte stores when the
// output base is 16-byte aligned, 4-byte stores otherwise).
__device__ __forceinline__ void store_row64(__half* dst, const float (&v)[64], float inv, bool vec) {
    if (vec) {
#pragma unroll
        for (int d = 0; d < 64; d += 8)
            *reinterpret_cast<uint4*>(dst + d) =
                make_uint4(pack_half2(v[d] * inv, v[d + 1] * inv),
                           pack_half2(v[d + 2] * inv, v[d + 3] * inv),
                           pack_half2(v[d + 4] * inv, v[d + 5] * inv),
                           pack_half2(v[d + 6] * inv, v[d + 7] * inv));
    } else {
#pragma unroll
        for (int d = 0; d < 64; d += 2)
            *reinterpret_cast<uint32_t*>(dst + d) = pack_half2(v[d] * inv, v[d + 1] * inv);
    }
}

template <int D, int STAGES>
__global__ void __launch_bounds__(192, 2) prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
    using S = PrefillTcSmem<D, STAGES>;
    constexpr int ROWS = S::kRows;
    constexpr int TILE = S::kTile;
    constexpr uint32_t kIdescS = umma_idesc_f16(ROWS, TILE, false, false);
    constexpr uint32_t kIdescPV = umma_idesc_f16(ROWS, D, false, true);

    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char* qs = smem + S::kQOffset;
    unsigned char* ks = smem + S::kKOffset;
    unsigned char* vs = smem + S::kVOffset;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* v_full = k_full + STAGES;
    uint64_t* k_empty = v_full + STAGES;
    uint64_t* v_empty = k_empty + STAGES;
    uint64_t* s_full = v_empty + STAGES;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_free + 1;
    uint64_t* pv_full = p_full + 1;
    uint64_t* done = pv_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::kNumBars);

    const int nq = (p.T + ROWS - 1) / ROWS;
    // Heads vary fastest in launch order; work units run longest query tile
    // first (longest-processing-time first).  Unit u of a head is chunk c of
    // query tile qt, enumerating tiles from the last and chunks in order.
    const int h = blockIdx.x;
    int qt = nq - 1, c = int(blockIdx.y), nc = 1, slot0 = 0;
    const int ct = p.chunk_tiles;
    for (;; --qt) {
        const int n = (min(qt * ROWS + ROWS, p.T) + TILE - 1) / TILE;
        nc = ct > 0 ? (n + ct - 1) / ct : 1;
        if (c < nc || qt == 0) break;
        c -= nc;
        if (nc > 1) slot0 += nc;
    }
    const int kvh = h / p.G;
    const int q0 = qt * ROWS;
    const int nkv_all = (min(q0 + ROWS, p.T) + TILE - 1) / TILE;
    const int j0 = nc > 1 ? c * ct : 0;                      // this unit's K/V tiles
    const int nkv = nc > 1 ? min(ct, nkv_all - j0) : nkv_all;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    grid_launch_dependents();
    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(pv_full, 1);
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, S::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_wait();

    if (warp == 4) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tensormap(&p.qmap);
            prefetch_tensormap(&p.kmap);
            prefetch_tensormap(&p.vmap);
            const uint64_t policy = l2_policy_evict_normal();
            mbar_arrive_expect_tx(q_full, uint32_t(S::kQBytes));
#pragma unroll
            for (int sub = 0; sub < S::kSub; ++sub)
#pragma unroll
                for (int half = 0; half < ROWS / TILE; ++half)
                    tma_load_4d(qs + sub * S::kQSubBytes + half * S::kKvSubBytes, &p.qmap, 0, sub,
                                h, q0 + half * TILE, q_full, policy);
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                const int s = j % STAGES;
                const uint32_t par = ((j / STAGES) - 1) & 1;
                if (j >= STAGES && !mbar_wait_bounded(&k_empty[s], par)) {
                    record_error(p.err, kDevTimeoutEmpty);
                    break;
                }
                mbar_arrive_expect_tx(&k_full[s], uint32_t(S::kKvBytes));
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub)
                    tma_load_4d(ks + s * S::kKvBytes + sub * S::kKvSubBytes, &p.kmap, 0, sub, kvh,
                                (j0 + j) * TILE, &k_full[s], policy);
                if (j >= STAGES && !mbar_wait_bounded(&v_empty[s], par)) {
                    record_error(p.err, kDevTimeoutEmpty);
                    mbar_arrive_expect_tx(&v_full[s], 0);
                    ++issued;
                    break;
                }
                mbar_arrive_expect_tx(&v_full[s], uint32_t(S::kKvBytes));
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub)
                    tma_load_4d(vs + s * S::kKvBytes + sub * S::kKvSubBytes, &p.vmap, 0, sub, kvh,
                                (j0 + j) * TILE, &v_full[s], policy);
                ++issued;
            }
            for (int j = max(0, issued - STAGES); j < issued; ++j) {
                const uint32_t par = (j / STAGES) & 1;
                if (!mbar_wait_bounded(&k_full[j % STAGES], par) ||
                    !mbar_wait_bounded(&v_full[j % STAGES], par)) {
                    record_error(p.err, kDevTimeoutFull);
                    break;
                }
            }
            if (!mbar_wait_bounded(q_full, 0)) record_error(p.err, kDevTimeoutFull);
        }
    } else if (warp == 5) {
        // ------------------------------------------------------ MMA issue
        if (lane == 0) {
            const uint32_t q_s = smem_u32(qs), k_s = smem_u32(ks), v_s = smem_u32(vs);
            const uint32_t t_o = tmem + S::kOCol;
            bool ok = mbar_wait_bounded(q_full, 0);
            auto issue_pv = [&](int i) -> bool {
                const int s = i % STAGES;
                if (!mbar_wait_bounded(&v_full[s], (i / STAGES) & 1) ||
                    !mbar_wait_bounded(p_full, i & 1))
                    return false;
                tc_fence_after();
                const uint32_t vt = v_s + s * S::kKvBytes;
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk) {
                    const uint64_t bd = umma_desc_sw128(vt + kk * 2048, S::kKvSubBytes, 1024);
                    umma_f16_ts(t_o, tmem + S::kPhiCol + kk * 8, bd, kIdescPV, i > 0 || kk > 0);
                    umma_f16_ts(t_o, tmem + S::kPloCol + kk * 8, bd, kIdescPV, true);
                }
                umma_commit(pv_full);
                umma_commit(&v_empty[s]);
                return true;
            };
            for (int j = 0; ok && j < nkv; ++j) {
                const int s = j % STAGES;
                if (!mbar_wait_bounded(&k_full[s], (j / STAGES) & 1) ||
                    (j > 0 && !mbar_wait_bounded(s_free, (j - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t kt = k_s + s * S::kKvBytes;
#pragma unroll
                for (int kc = 0; kc < D / 16; ++kc) {
                    const int sub = kc / 4, c = kc % 4;
                    umma_f16(tmem,
                             umma_desc_sw128(q_s + sub * S::kQSubBytes + c * 32, 16, 1024),
                             umma_desc_sw128(kt + sub * S::kKvSubBytes + c * 32, 16, 1024),
                             kIdescS, kc > 0);
                }
                umma_commit(s_full);
                umma_commit(&k_empty[s]);
                if (j > 0 && !issue_pv(j - 1)) ok = false;
            }
            if (ok && !issue_pv(nkv - 1)) ok = false;
            if (!ok) record_error(p.err, kDevTimeoutFull);
            umma_commit(done);
            if (!mbar_wait_bounded(done, 0)) record_error(p.err, kDevTimeoutFull);
        }
    } else {
        // --------------------------------------------------------- softmax
        const int r = threadIdx.x;
        const int qrow = q0 + r;
        const uint32_t lane_base = uint32_t(warp * 32) << 16;
        const uint32_t t_row = tmem + lane_base;
        const float sl2 = p.scale_log2;
        float m_ref = -INFINITY, l_run = 0.f;
        bool ok = true;

        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait_bounded(s_full, j & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[64];
            tmem_ld64(t_row, sv);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);

            const int key0 = (j0 + j) * TILE;
            if (key0 + TILE - 1 > q0 || key0 + TILE > p.T) {
#pragma unroll
                for (int c = 0; c < TILE; ++c)
                    if (key0 + c > qrow || key0 + c >= p.T) sv[c] = -INFINITY;
            }
            // 8 independent partial maxima / sums: short dependency chains
            float pm[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) pm[i] = sv[i];
#pragma unroll
            for (int c = 8; c < TILE; ++c) pm[c & 7] = fmaxf(pm[c & 7], sv[c]);
            float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
            mx *= sl2;
            float alpha = 1.f;
            if (mx > m_ref + kRescaleLog2) {
                alpha = fast_exp2(m_ref - mx);          // 0 on the first tile
                m_ref = mx;
            }
            const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
            float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            uint32_t hw[32], lw[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float a = fast_exp2(fmaf(sv[2 * c], sl2, -m_use));
                const float b = fast_exp2(fmaf(sv[2 * c + 1], sl2, -m_use));
                ps[c & 7] += a + b;
                const float ah = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
                const float bh = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
                hw[c] = pack_half2(ah, bh);
                lw[c] = pack_half2(a - ah, b - bh);
            }
            const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            l_run = fmaf(l_run, alpha, rs);

            if (j > 0) {
                // PV_{j-1} complete: P may be overwritten and O is current
                if (!mbar_wait_bounded(pv_full, (j - 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                    for (int c0 = 0; c0 < D; c0 += 32) {
                        float ov[32];
                        tmem_ld32(t_row + S::kOCol + c0, ov);
                        uint32_t w[32];
#pragma unroll
                        for (int c = 0; c < 32; ++c) w[c] = __float_as_uint(ov[c] * alpha);
                        tmem_st32(t_row + S::kOCol + c0, w);
                    }
                }
            }
            tmem_st32(t_row + S::kPhiCol, hw);
            tmem_st32(t_row + S::kPloCol, lw);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && !mbar_wait_bounded(pv_full, (nkv - 1) & 1)) ok = false;
        if (!ok) record_error(p.err, kDevTimeoutFull);
        __half* dst = p.out + ((size_t)qrow * p.H + h) * D;
        const bool vec = (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
        if (ok && nc == 1) {
            tc_fence_after();
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 64) {
                float ov[64];
                tmem_ld64(t_row + S::kOCol + c0, ov);   // whole warp, rows past T included
                if (qrow < p.T) store_row64(dst + c0, ov, inv, vec);
            }
        } else if (nc > 1) {
            // Split K/V range: store this unit's unnormalised row state
            // (O d-major, [d][row], so a warp's stores and loads are whole
            // 128-byte lines); the last unit of the query tile to arrive
            // merges the others into its own state, read back from TMEM.
            const size_t slot0g = (size_t)h * p.slots_per_head + slot0;
            float2* mlp = reinterpret_cast<float2*>(p.part_ml) + slot0g * ROWS + r;
            if (ok) {
                tc_fence_after();
                float* pa = p.part_acc + (slot0g + c) * ROWS * D + r;
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 64) {
                    float ov[64];
                    tmem_ld64(t_row + S::kOCol + c0, ov);
#pragma unroll
                    for (int d = 0; d < 64; ++d) pa[(c0 + d) * ROWS] = ov[d];
                }
                mlp[c * ROWS] = make_float2(m_ref, l_run);
            }
            uint32_t* last = tmem_slot + 1;
            consumer_sync(4 * 32);                   // this unit's stores are done
            if (threadIdx.x == 0) {
                // acq_rel: publishes this unit's state and, for the last
                // arriver, acquires the other units' states.
                const int old = atom_add_acq_rel_gpu(&p.counters[h * nq + qt], 1);
                *last = (old == nc - 1) ? 1u : 0u;
            }
            consumer_sync(4 * 32);
            if (*last && ok) {
                // O = sum_u O_u 2^(m_u - M) / sum_u l_u 2^(m_u - M), M = max_u m_u
                float mu_[kMaxPrefillChunks], lu_[kMaxPrefillChunks];
                float mmax = m_ref;
#pragma unroll
                for (int u = 0; u < kMaxPrefillChunks; ++u) {
                    mu_[u] = -INFINITY;
                    lu_[u] = 0.f;
                    if (u < nc && u != c) {
                        const float2 v = __ldcg(mlp + u * ROWS);
                        mu_[u] = v.x;
                        lu_[u] = v.y;
                    }
                    mmax = fmaxf(mmax, mu_[u]);
                }
                const float msafe = mmax == -INFINITY ? 0.f : mmax;
                const float w_own = fast_exp2(m_ref - msafe);
                float lsum = l_run * w_own;
#pragma unroll
                for (int u = 0; u < kMaxPrefillChunks; ++u) {
                    mu_[u] = fast_exp2(mu_[u] - msafe);          // weight (0 for absent units)
                    lsum = fmaf(lu_[u], mu_[u], lsum);
                }
                const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 64) {
                    float ov[64];
                    tmem_ld64(t_row + S::kOCol + c0, ov);        // whole warp
#pragma unroll
                    for (int d = 0; d < 64; ++d) ov[d] *= w_own;
#pragma unroll
                    for (int u = 0; u < kMaxPrefillChunks; ++u) {
                        if (u < nc && u != c) {
                            const float* src = p.part_acc + ((slot0g + u) * D + c0) * ROWS + r;
#pragma unroll
                            for (int d = 0; d < 64; ++d)
                                ov[d] = fmaf(__ldcg(src + d * ROWS), mu_[u], ov[d]);
                        }
                    }
                    if (qrow < p.T) store_row64(dst + c0, ov, inv, vec);
                }
            }
            if (*last && threadIdx.x == 0) p.counters[h * nq + qt] = 0;   // ready for the next call
        }
        tc_fence_before();
    }

    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

}  // namespace fr
