// prefill_tc_kernels.cuh - causal prefill attention on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// Same contract and result as prefill_kernel (prefill_kernels.cuh), which it
// replaces as the default path of fr_prefill_attn: prefill_attn_causal
// (kernels/attention.cuh:76-82, kernels/attention_decode.cu:563-619), query
// position s of head h attends to positions 0..s of kv head h / (H / Hkv),
// scale 1/sqrt(D), fp32 softmax and accumulation, one fp16 rounding.
//
// One CTA per (128-row query tile, query head), 192 threads:
//   warps 0-3  softmax: thread r owns query row r of the tile (TMEM lane r);
//   warp 4     producer: TMA loads of the Q tile and of the causal K/V tiles
//              (64 positions x D, 128-byte swizzle) through a STAGES ring;
//   warp 5     allocates tensor memory; its lane 0 issues every tcgen05.mma.
// Per K/V tile j:
//   S_j = Q K_j^T            M=128, N=64, K=D; Q and K both K-major from the
//                            TMA tiles; fp32 into TMEM columns [0, 64);
//   softmax                  each thread reads its row of S_j (tcgen05.ld),
//                            masks, updates the base-2 online softmax and
//                            writes P_j as an fp16 pair (hi + lo, ~22 bits)
//                            into shared memory in the 128-byte-swizzled
//                            K-major layout of an MMA A operand;
//   PV_j = P_j V_j           M=128, N=D, K=64 (hi and lo accumulate into the
//                            same TMEM tile); V is the MN-major B operand read
//                            straight from the TMA tile; two TMEM buffers
//                            alternate so PV_j runs while the softmax warps
//                            fold PV_{j-1} into their register accumulator:
//                            O = (O + PV_{j-1}) * 2^(m_{j-1} - m_j).
// The tensor pipe runs S_{j+1} as soon as the softmax warps have read S_j.
// Every wait is bounded; on a timeout the kernel records an error, stops
// issuing, waits for its own MMAs and copies and frees tensor memory.
#pragma once
#include "decode_kernels.cuh"
#include "prefill_kernels.cuh"
#include "tc_ptx.cuh"

namespace fr {

template <int D, int STAGES>
struct PrefillTcSmem {
    static constexpr int kRows = 128;                       // query rows per CTA (MMA M)
    static constexpr int kTile = 64;                        // K/V positions per tile (MMA N of S)
    static constexpr int kSub = D / 64;                     // 128-byte column blocks of D
    static constexpr int kQSubBytes = kRows * 128;          // [128 rows][64 dims]
    static constexpr int kQBytes = kSub * kQSubBytes;
    static constexpr int kKvSubBytes = kTile * 128;         // [64 positions][64 dims]
    static constexpr int kKvBytes = kSub * kKvSubBytes;
    static constexpr int kPBytes = kRows * 128;             // [128 rows][64 positions] fp16
    static constexpr size_t kQOffset = 0;
    static constexpr size_t kKOffset = kQBytes;
    static constexpr size_t kVOffset = kKOffset + size_t(STAGES) * kKvBytes;
    static constexpr size_t kPOffset = kVOffset + size_t(STAGES) * kKvBytes;  // hi, then lo
    static constexpr size_t kBarOffset = kPOffset + 2 * size_t(kPBytes);
    // barriers: q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full,
    // s_free, p_full, pv_full[2], done; then the TMEM base address slot
    static constexpr int kNumBars = 1 + 4 * STAGES + 6;
    static constexpr size_t kBytes = 1024 + kBarOffset + kNumBars * sizeof(uint64_t) + 16;
    // TMEM columns: S at [0, 64), PV buffer b at kPvCol + b * D
    static constexpr uint32_t kPvCol = D >= 128 ? 128 : 64;
    static constexpr uint32_t kTmemCols = (kPvCol + 2 * D) <= 256 ? 256 : 512;
};

template <int D, int STAGES>
__global__ void __launch_bounds__(192, 1) prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
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
    unsigned char* ps = smem + S::kPOffset;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* v_full = k_full + STAGES;
    uint64_t* k_empty = v_full + STAGES;
    uint64_t* v_empty = k_empty + STAGES;
    uint64_t* s_full = v_empty + STAGES;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_free + 1;
    uint64_t* pv_full = p_full + 1;          // [2]
    uint64_t* done = pv_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::kNumBars);

    const int nq = (p.T + ROWS - 1) / ROWS;
    const int qt = nq - 1 - int(blockIdx.x);  // longest first
    const int h = blockIdx.y;
    const int kvh = h / p.G;
    const int q0 = qt * ROWS;
    const int nkv = (min(q0 + ROWS, p.T) + TILE - 1) / TILE;  // causal K/V tiles
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
        mbar_init(&pv_full[0], 1);
        mbar_init(&pv_full[1], 1);
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
    grid_dependency_wait();                   // q, k, v may come from the preceding grid

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
                                j * TILE, &k_full[s], policy);
                if (j >= STAGES && !mbar_wait_bounded(&v_empty[s], par)) {
                    // K was issued: count this tile so its copy is drained
                    record_error(p.err, kDevTimeoutEmpty);
                    mbar_arrive_expect_tx(&v_full[s], 0);
                    ++issued;
                    break;
                }
                mbar_arrive_expect_tx(&v_full[s], uint32_t(S::kKvBytes));
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub)
                    tma_load_4d(vs + s * S::kKvBytes + sub * S::kKvSubBytes, &p.vmap, 0, sub, kvh,
                                j * TILE, &v_full[s], policy);
                ++issued;
            }
            // Drain: no copy in flight at exit.
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
            const uint32_t phi = smem_u32(ps), plo = phi + S::kPBytes;
            const uint32_t t_s = tmem;
            bool ok = mbar_wait_bounded(q_full, 0);
            // PV_i = P_i V_i into TMEM buffer i % 2 (hi then lo, same accumulator)
            auto issue_pv = [&](int i) -> bool {
                const int s = i % STAGES;
                if (!mbar_wait_bounded(&v_full[s], (i / STAGES) & 1) ||
                    !mbar_wait_bounded(p_full, i & 1))
                    return false;
                tc_fence_after();
                const uint32_t t_pv = tmem + S::kPvCol + uint32_t(i & 1) * D;
                const uint32_t vt = v_s + s * S::kKvBytes;
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk) {
                    const uint64_t bd = umma_desc_sw128(vt + kk * 2048, S::kKvSubBytes, 1024);
                    umma_f16(t_pv, umma_desc_sw128(phi + kk * 32, 16, 1024), bd, kIdescPV, kk > 0);
                    umma_f16(t_pv, umma_desc_sw128(plo + kk * 32, 16, 1024), bd, kIdescPV, true);
                }
                umma_commit(&pv_full[i & 1]);
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
                    umma_f16(t_s,
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
            // every MMA issued above has completed before tensor memory is freed
            umma_commit(done);
            if (!mbar_wait_bounded(done, 0)) record_error(p.err, kDevTimeoutFull);
        }
    } else {
        // --------------------------------------------------------- softmax
        const int r = threadIdx.x;                       // tile row = TMEM lane
        const int qrow = q0 + r;
        const uint32_t lane_base = uint32_t(warp * 32) << 16;
        const uint32_t t_s = tmem + lane_base;
        unsigned char* prow_hi = ps + r * 128;
        unsigned char* prow_lo = prow_hi + S::kPBytes;
        const int sw = r & 7;
        const float sl2 = p.scale_log2;
        float o[D];
#pragma unroll
        for (int d = 0; d < D; ++d) o[d] = 0.f;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;

        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait_bounded(s_full, j & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[64];
            tmem_ld64(t_s, sv);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);

            const int key0 = j * TILE;
            if (key0 + TILE - 1 > q0 || key0 + TILE > p.T) {
#pragma unroll
                for (int c = 0; c < TILE; ++c)
                    if (key0 + c > qrow || key0 + c >= p.T) sv[c] = -INFINITY;
            }
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < TILE; ++c) mx = fmaxf(mx, sv[c]);
            const float m_new = fmaxf(m_run, mx * sl2);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = fast_exp2(m_run - m_use);
            m_run = m_new;
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < TILE; ++c) {
                sv[c] = fast_exp2(fmaf(sv[c], sl2, -m_use));
                rs += sv[c];
            }
            l_run = fmaf(l_run, alpha, rs);

            // P_{j-1} is no longer read once PV_{j-1} has completed
            if (j > 0 && !mbar_wait_bounded(&pv_full[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
                ok = false;
                break;
            }
            // P_j = hi + lo: hi keeps the top 11 significant bits (exact in
            // fp16 for p >= 2^-14), lo the exact fp32 remainder.
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a = sv[8 * c + 2 * e], b = sv[8 * c + 2 * e + 1];
                    const float ah = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
                    const float bh = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
                    hw[e] = pack_half2(ah, bh);
                    lw[e] = pack_half2(a - ah, b - bh);
                }
                const int off = ((c ^ sw) << 4);
                *reinterpret_cast<uint4*>(prow_hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(prow_lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);

            // O = (O + PV_{j-1}) * alpha while PV_j runs in the other buffer
            if (j > 0) {
                tc_fence_after();
                const uint32_t t_pv = tmem + lane_base + S::kPvCol + uint32_t((j - 1) & 1) * D;
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 64) {
                    float pv[64];
                    tmem_ld64(t_pv + c0, pv);
#pragma unroll
                    for (int c = 0; c < 64; ++c) o[c0 + c] = (o[c0 + c] + pv[c]) * alpha;
                }
            }
        }
        if (ok) {
            const int last = nkv - 1;
            if (!mbar_wait_bounded(&pv_full[last & 1], (last >> 1) & 1)) {
                ok = false;
            } else {
                tc_fence_after();
                const uint32_t t_pv = tmem + lane_base + S::kPvCol + uint32_t(last & 1) * D;
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 64) {
                    float pv[64];
                    tmem_ld64(t_pv + c0, pv);
#pragma unroll
                    for (int c = 0; c < 64; ++c) o[c0 + c] += pv[c];
                }
            }
        }
        if (!ok) record_error(p.err, kDevTimeoutFull);
        if (ok && qrow < p.T) {
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            __half* dst = p.out + ((size_t)qrow * p.H + h) * D;
            if ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0) {
#pragma unroll
                for (int d = 0; d < D; d += 8)
                    *reinterpret_cast<uint4*>(dst + d) =
                        make_uint4(pack_half2(o[d] * inv, o[d + 1] * inv),
                                   pack_half2(o[d + 2] * inv, o[d + 3] * inv),
                                   pack_half2(o[d + 4] * inv, o[d + 5] * inv),
                                   pack_half2(o[d + 6] * inv, o[d + 7] * inv));
            } else {
#pragma unroll
                for (int d = 0; d < D; d += 2)
                    *reinterpret_cast<uint32_t*>(dst + d) = pack_half2(o[d] * inv, o[d + 1] * inv);
            }
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
