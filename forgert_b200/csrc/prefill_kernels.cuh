// prefill_kernels.cuh - causal prefill attention (fr_prefill_attn).
//
// Replaces prefill_attn_causal (kernels/attention.cuh:76-82, definition
// kernels/attention_decode.cu:563-619), which runs one thread per (head,
// query position) over that position's prefix.  Same result: query position
// s of head h attends to positions 0..s of kv head h / (H / Hkv), softmax
// scale 1/sqrt(D), fp32 softmax and accumulation, one fp16 rounding.
//
// Flash-attention form on the tensor cores: one CTA per (64-row query tile,
// query head); warps 0-3 own 16 query rows each, warp 4 is the producer.  The
// producer TMA-loads the query tile once and streams the causal K/V tiles
// (64 positions x D, the same tensor-map boxes and 128-byte swizzle as the
// decode kernel) through a STAGES-deep mbarrier ring.  Per K/V tile a warp
// computes S = Q K^T (mma.sync m16n8k16: Q as the A operand from registers,
// K rows as B fragments through ldmatrix), masks the causal diagonal and the
// rows past T, updates the online softmax in base 2, and accumulates
// O += P V with P taken straight from the S accumulator layout (which is the
// A-fragment layout) and V rows as B fragments through ldmatrix.trans.  P
// enters P.V as an fp16 pair (hi + lo), ~22 bits, like the decode kernel.
// Query tiles are launched longest first (the last tile needs the most K/V).
#pragma once
#include "decode_kernels.cuh"

namespace fr {

struct PrefillParams {
    CUtensorMap qmap;            // Q view [T][H][D/64][64], box 64 dims x 64 rows
    CUtensorMap kmap;            // K view [T][Hkv][D/64][64]
    CUtensorMap vmap;            // V view, same geometry
    __half* out;                 // [T, H, D]
    int T, H, Hkv, G;            // positions, query heads, kv heads, H / Hkv
    float scale_log2;            // log2(e) / sqrt(D)
    int* err;                    // device error word
    // Split K/V ranges (tcgen05 kernel only; chunk_tiles == 0: one CTA per
    // query tile).  A query tile with more than chunk_tiles K/V tiles is
    // covered by several CTAs; each stores its unnormalised (O, m, l) in
    // slot h * slots_per_head + (the tile's first slot) + chunk, and the last
    // to arrive (counters[h * nq + query tile]) merges them.
    int chunk_tiles;
    int slots_per_head;
    float* part_acc;             // [slots][D][128 rows]
    float* part_ml;              // [slots][128 rows][2]
    int* counters;               // zero between calls
};

template <int D, int STAGES>
struct PrefillSmem {
    static constexpr int kTile = 64;                               // rows per tile
    static constexpr int kSub = D / 64;                            // 128-byte column blocks
    static constexpr int kSubBytes = kTile * 128;                  // one [64][64] box
    static constexpr int kTileBytes = kSub * kSubBytes;            // 64 rows x D
    static constexpr size_t kQOffset = 0;
    static constexpr size_t kRingOffset = kTileBytes;              // K stages, then V stages
    static constexpr size_t kBarOffset = kRingOffset + size_t(2) * STAGES * kTileBytes;
    // +1024: realignment of the dynamic shared memory to the swizzle atom.
    static constexpr size_t kBytes = 1024 + kBarOffset + (2 * STAGES + 1) * sizeof(uint64_t);
};

// grid = (H, ceil(T / 64) query tiles), block = 160 (4 consumer warps + producer).
template <int D, int STAGES>
__global__ void __launch_bounds__(160) prefill_kernel(const __grid_constant__ PrefillParams p) {
    using S = PrefillSmem<D, STAGES>;
    constexpr int NW = 4;
    constexpr int TILE = S::kTile;
    constexpr int KSTEPS = D / 16;          // k-steps of Q K^T
    constexpr int DN = D / 8;               // 8-column n-tiles of O
    constexpr int SN = TILE / 8;            // 8-key n-tiles of S

    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char* qs = smem + S::kQOffset;
    unsigned char* kring = smem + S::kRingOffset;
    unsigned char* vring = kring + STAGES * S::kTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* qbar = empty + STAGES;

    const int nq = (p.T + TILE - 1) / TILE;
    // Heads vary fastest in launch order: every head's longest query tile
    // is scheduled before any shorter one (longest-processing-time first).
    const int h = blockIdx.x;
    const int qt = nq - 1 - int(blockIdx.y);
    const int kvh = h / p.G;
    const int q0 = qt * TILE;
    const int nkv = qt + 1;                    // causal: K/V tiles 0..qt
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    grid_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        mbar_init(qbar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NW) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tensormap(&p.qmap);
            prefetch_tensormap(&p.kmap);
            prefetch_tensormap(&p.vmap);
            // K/V tiles are read again by later query tiles and the other
            // heads of the group: keep them in L2 (normal priority).
            const uint64_t policy = l2_policy_evict_normal();
            grid_dependency_wait();             // q, k, v may come from the preceding grid
            mbar_arrive_expect_tx(qbar, uint32_t(S::kTileBytes));
#pragma unroll
            for (int sub = 0; sub < S::kSub; ++sub)
                tma_load_4d(qs + sub * S::kSubBytes, &p.qmap, 0, sub, h, q0, qbar, policy);
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                const int s = j % STAGES;
                if (j >= STAGES && !mbar_wait_bounded(&empty[s], ((j / STAGES) - 1) & 1)) {
                    record_error(p.err, kDevTimeoutEmpty);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], uint32_t(2 * S::kTileBytes));
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub) {
                    tma_load_4d(kring + s * S::kTileBytes + sub * S::kSubBytes, &p.kmap, 0, sub,
                                kvh, j * TILE, &full[s], policy);
                    tma_load_4d(vring + s * S::kTileBytes + sub * S::kSubBytes, &p.vmap, 0, sub,
                                kvh, j * TILE, &full[s], policy);
                }
                ++issued;
            }
            // Drain: no copy in flight at exit.
            for (int j = max(0, issued - STAGES); j < issued; ++j) {
                if (!mbar_wait_bounded(&full[j % STAGES], (j / STAGES) & 1)) {
                    record_error(p.err, kDevTimeoutFull);
                    break;
                }
            }
            if (!mbar_wait_bounded(qbar, 0)) record_error(p.err, kDevTimeoutFull);
        }
        __syncwarp();
        return;
    }

    // --------------------------------------------------------- consumers
    grid_dependency_wait();
    const int g = lane >> 2;
    const int t = lane & 3;
    if (!mbar_wait_bounded(qbar, 0)) {
        record_error(p.err, kDevTimeoutFull);
        return;
    }
    // Q rows 16*warp .. +15 as A fragments: a0 (rows 0-7, k 0-7), a1 (rows
    // 8-15, k 0-7), a2 (rows 0-7, k 8-15), a3 (rows 8-15, k 8-15).
    uint32_t qa[KSTEPS][4];
    {
        const uint32_t qs_s = smem_u32(qs);
        const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = ((lane >> 4) & 1) * 8;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks)
            ldsm_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3],
                    qs_s + swz_offset<TILE>(row, ks * 16 + col));
    }

    float o[DN][4];
#pragma unroll
    for (int dn = 0; dn < DN; ++dn)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[dn][c] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};
    const int row_lo = q0 + warp * 16 + g;     // query positions of this lane's two rows
    const int row_hi = row_lo + 8;
    const float sl2 = p.scale_log2;
    const uint32_t kring_s = smem_u32(kring);
    const uint32_t vring_s = smem_u32(vring);
    // ldmatrix rows/columns of this lane for the K (non-transposed) and V
    // (transposed) B fragments.
    const int k_row = (lane & 7) + ((lane >> 4) & 1) * 8;
    const int k_col = ((lane >> 3) & 1) * 8;
    const int v_row = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int v_col = ((lane >> 4) & 1) * 8;
    bool ok = true;

    for (int j = 0; j < nkv; ++j) {
        const int s = j % STAGES;
        if (!mbar_wait_bounded(&full[s], (j / STAGES) & 1)) {
            record_error(p.err, kDevTimeoutFull);
            ok = false;
            break;
        }
        const uint32_t kst = kring_s + s * S::kTileBytes;
        const uint32_t vst = vring_s + s * S::kTileBytes;

        // ---- S = Q K^T (16 rows x 64 keys): n-tile n covers keys 8n..8n+7
        float sacc[SN][4];
#pragma unroll
        for (int n = 0; n < SN; ++n)
#pragma unroll
            for (int c = 0; c < 4; ++c) sacc[n][c] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
            for (int np = 0; np < SN / 2; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, kst + swz_offset<TILE>(np * 16 + k_row, ks * 16 + k_col));
                mma_16816(sacc[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
                mma_16816(sacc[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
            }
        }

        // ---- causal mask on the diagonal tile, and keys past T
        const int key0 = j * TILE;
        if (j == qt || key0 + TILE > p.T) {
#pragma unroll
            for (int n = 0; n < SN; ++n) {
                const int key = key0 + n * 8 + 2 * t;
                if (key > row_lo || key >= p.T) sacc[n][0] = -INFINITY;
                if (key + 1 > row_lo || key + 1 >= p.T) sacc[n][1] = -INFINITY;
                if (key > row_hi || key >= p.T) sacc[n][2] = -INFINITY;
                if (key + 1 > row_hi || key + 1 >= p.T) sacc[n][3] = -INFINITY;
            }
        }

        // ---- online softmax per row (base 2); the 4 lanes of a row share it
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < SN; ++n) {
            mx[0] = fmaxf(mx[0], fmaxf(sacc[n][0], sacc[n][1]));
            mx[1] = fmaxf(mx[1], fmaxf(sacc[n][2], sacc[n][3]));
        }
        float alpha[2], m_use[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float m_new = fmaxf(m_run[r], mx[r] * sl2);
            m_use[r] = (m_new == -INFINITY) ? 0.f : m_new;
            alpha[r] = fast_exp2(m_run[r] - m_use[r]);
            m_run[r] = m_new;
        }
        float rs[2] = {0.f, 0.f};
#pragma unroll
        for (int n = 0; n < SN; ++n) {
            sacc[n][0] = fast_exp2(fmaf(sacc[n][0], sl2, -m_use[0]));
            sacc[n][1] = fast_exp2(fmaf(sacc[n][1], sl2, -m_use[0]));
            sacc[n][2] = fast_exp2(fmaf(sacc[n][2], sl2, -m_use[1]));
            sacc[n][3] = fast_exp2(fmaf(sacc[n][3], sl2, -m_use[1]));
            rs[0] += sacc[n][0] + sacc[n][1];
            rs[1] += sacc[n][2] + sacc[n][3];
        }
        l_run[0] = fmaf(l_run[0], alpha[0], rs[0]);
        l_run[1] = fmaf(l_run[1], alpha[1], rs[1]);
#pragma unroll
        for (int dn = 0; dn < DN; ++dn) {
            o[dn][0] *= alpha[0];
            o[dn][1] *= alpha[0];
            o[dn][2] *= alpha[1];
            o[dn][3] *= alpha[1];
        }

        // ---- O += P V: k-step kk covers keys 16kk..16kk+15 = S n-tiles 2kk, 2kk+1
#pragma unroll
        for (int kk = 0; kk < TILE / 16; ++kk) {
            const float* p0 = sacc[2 * kk];
            const float* p1 = sacc[2 * kk + 1];
            const __half2 h0 = __floats2half2_rn(p0[0], p0[1]);
            const __half2 h1 = __floats2half2_rn(p0[2], p0[3]);
            const __half2 h2 = __floats2half2_rn(p1[0], p1[1]);
            const __half2 h3 = __floats2half2_rn(p1[2], p1[3]);
            const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&h0);
            const uint32_t a1 = *reinterpret_cast<const uint32_t*>(&h1);
            const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&h2);
            const uint32_t a3 = *reinterpret_cast<const uint32_t*>(&h3);
            const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
            const float2 f2 = __half22float2(h2), f3 = __half22float2(h3);
            const uint32_t l0 = pack_half2(p0[0] - f0.x, p0[1] - f0.y);
            const uint32_t l1 = pack_half2(p0[2] - f1.x, p0[3] - f1.y);
            const uint32_t l2 = pack_half2(p1[0] - f2.x, p1[1] - f2.y);
            const uint32_t l3 = pack_half2(p1[2] - f3.x, p1[3] - f3.y);
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(b0, b1, b2, b3, vst + swz_offset<TILE>(kk * 16 + v_row, dp * 16 + v_col));
                mma_16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
                mma_16816(o[2 * dp], l0, l1, l2, l3, b0, b1);
                mma_16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
                mma_16816(o[2 * dp + 1], l0, l1, l2, l3, b2, b3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!ok) return;

    // ---- normalise and store: lane holds rows (g, g + 8), columns 8dn + 2t, +1
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
    }
    const float l_lo = l_run[0], l_hi = l_run[1];
#pragma unroll
    for (int dn = 0; dn < DN; ++dn) {
        const int d = dn * 8 + 2 * t;
        if (row_lo < p.T)
            *reinterpret_cast<__half2*>(p.out + ((size_t)row_lo * p.H + h) * D + d) =
                __floats2half2_rn(l_lo > 0.f ? o[dn][0] / l_lo : 0.f,
                                  l_lo > 0.f ? o[dn][1] / l_lo : 0.f);
        if (row_hi < p.T)
            *reinterpret_cast<__half2*>(p.out + ((size_t)row_hi * p.H + h) * D + d) =
                __floats2half2_rn(l_hi > 0.f ? o[dn][2] / l_hi : 0.f,
                                  l_hi > 0.f ? o[dn][3] / l_hi : 0.f);
    }
}

}  // namespace fr
