// decode_kernels.cuh - split-KV flash-decode attention for sm_100a.
//
// Replaces the per-q-head SIMT kernel `decode_attn_kernel_v4<D,4>`
// (kernels/attention_decode.cu:418-533 of the reference), which launches one
// CTA per query head, re-reads each KV head G times and walks all of kv_len
// in one CTA.
//
// Work decomposition: one CTA per (sequence b, kv head, head group, KV split).
// The CTA serves the whole GQA query group of its kv head (up to 16 query
// heads), so every K/V byte is read from HBM exactly once per call.
//
// Data movement: warp NW (the producer) streams K and V tiles of TILE
// positions x 64 head dims into shared memory with 4-D TMA tensor copies
// (cp.async.bulk.tensor, each load into this CTA only): the tensor map views a cache as
// [rows][kv_heads][D/64][64] fp16, one box = 64 dims x TILE rows of one kv
// head, written with the 128-byte swizzle (16-byte chunk c of row r lands at
// chunk c ^ (r & 7)), which makes the ldmatrix reads below conflict-free.
// Tiles cycle through a STAGES-deep ring guarded by full/empty mbarriers.
// Rows past the end of the cache come back from TMA as zeros.
//
// Math: the NW consumer warps take 16 positions each of every tile and use
// the tensor cores with the query group as the N dimension:
//     S^T[pos, head]  = K[pos, :] . Q^T[:, head]      (mma m16n8k16, M = pos)
//     O^T[d, head]   += V^T[d, pos] . P^T[pos, head]  (mma m16n8k16, M = d)
// Q (fp16, exact) stays in registers as the B operand for the whole call;
// scores and the online softmax state (m, l) are fp32 in the base-2 domain
// (scale * log2 e folded into one multiply).  Each probability enters the
// P.V product as two fp16 halves (P = P_hi + P_lo), so the product keeps
// about 22 bits of P and matches the reference's fp32 P.V to fp32 rounding;
// accumulation is fp32.  P^T reaches the B-operand layout through
// movmatrix.trans, without a shared-memory round trip.
//
// Output: with one split the CTA normalises and writes fp16 directly.  With
// several, the CTAs of a thread-block cluster merge their (m, l, acc[D])
// states through distributed shared memory and the last cluster of each
// (sequence, kv head) merges the cluster partials (the flash-decoding
// log-sum-exp merge, fused into the same kernel); `lse_merge_kernel` is the
// separate-launch form of the same merge.
#pragma once
#include "fr_ptx.cuh"
#include "trace.cuh"
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cfloat>

namespace fr {

constexpr int kMaxRanks = 8;        // GPUs of one cross-GPU exchange

struct DecodeParams {
    CUtensorMap kmap;            // K view [rows][Hkv][D/64][64] (see file header)
    CUtensorMap vmap;            // V view, same geometry
    const __half* q;             // [B, H, D]
    const long long* row_offsets;// [B] first tensor-map row of each sequence, or nullptr (0)
    const int* kv_lens;          // [B] per-sequence lengths, or nullptr (use kv_len)
    int kv_len;
    int zero_tail;               // 1: rows past a sequence's end may hold non-finite data
    int prefetch_rows;           // rows [0, prefetch_rows) may be loaded before the grid
                                 // dependency wait (they are not written by the preceding
                                 // kernels); 0 = everything waits
    int H, Hkv, G;               // query heads, kv heads, group size H / Hkv
    int split_len;               // positions per split (multiple of TILE)
    int num_splits;              // gridDim.y
    int head_groups;             // gridDim.x / Hkv
    float scale_log2;            // log2(e) / sqrt(D)
    int write_final;             // 1: single split, write normalised fp16 to out
    __half* out;                 // [B, H, D]
    float* out_ml;               // non-null: write merged states (m, l) [B*H, 2] instead of out
    float* out_acc;              //           and acc [B*H, D]
    float* part_ml;              // partial states, slot (row * part_slots + j): (m, l)
    float* part_acc;             //                                            acc[D]
    int part_slots;              // slots per row: num_splits (unfused) or num_splits / CL
    int* counters;               // fused merge: one per (b, kv head, head group), zero
                                 // between calls; nullptr = unfused (lse_merge_kernel follows)
    int* err;                    // device error word
    int evict_normal;            // 1: K/V loads without the L2 evict-first hint
    // Persistent batched kernel (batched_kernels.cuh): sequences of the call
    // and whether lengths, row offsets and all but each unit's last tile may
    // be read before the grid-dependency wait.
    int batch;
    int prefetch_meta;
    // The persistent grid uses only as many CTAs as give each at least
    // min_tiles_per_cta tiles, never fewer than min_ctas (0 = all of them).
    int min_tiles_per_cta;
    int min_ctas;
    // Cost map of the persistent partition (tile-times): per unit, item_cost
    // before its first tile and merge_cost after its last.
    int item_cost;
    int merge_cost;
    // Paged KV (kernel instantiated with PAGED): the tensor maps view the page
    // pool [num_pages * page_size rows][Hkv][D/64][64]; logical position t of
    // sequence b is row block_table[b * bt_stride + t / page_size] * page_size
    // + t % page_size.
    const int* block_table;      // [B, bt_stride] page ids
    int bt_stride;               // entries per block-table row
    int page_size;               // rows per page, multiple of 16
    int page_box;                // rows per TMA box: gcd(page_size, TILE)
    int num_pages;               // pool size; other ids read as zeros
    // Cross-GPU exchange (xworld > 0, fused path only): the final (m, l, acc)
    // state slices go to every rank's exchange buffer (XLayout) and each rank
    // merges the xworld states of every head row into `out`.
    void* xbuf[kMaxRanks];       // exchange buffer of each rank ([xrank] = this GPU's)
    int xrank, xworld;
    int xrows;                   // head rows per state (B * H)
    int xwait_ms;                // longest wait for the other ranks' words (ms)
};

// Layout of one rank's exchange buffer (bytes from its base):
//   [0, 256)   header: u32 epoch (calls completed), u32 count (CTAs of the
//              current call that have read the epoch)
//   then ml  [2 parities][world][rows][2] u64 words
//   then acc [2 parities][world][rows][D] u64 words
// Every word is (epoch of the call that wrote it) << 32 | fp32 bits, stored
// by the source rank in one 8-byte access; the reader waits until a word's
// tag equals its own epoch.  Call e uses parity e & 1; a rank can start call
// e + 2 only after every rank finished call e + 1, so a parity is never
// overwritten while it is read.  All zero (tag 0) is "nothing written".
struct XLayout {
    static constexpr size_t kHeader = 256;
    __host__ __device__ static size_t bytes(int world, int rows, int D) {
        return kHeader + size_t(2) * world * rows * (2 + D) * sizeof(uint64_t);
    }
    __host__ __device__ static uint32_t* header(void* base) {
        return reinterpret_cast<uint32_t*>(base);
    }
    __host__ __device__ static uint64_t* ml(void* base, int par, int src, int world, int rows) {
        uint64_t* m0 = reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(base) + kHeader);
        return m0 + (size_t)(par * world + src) * rows * 2;
    }
    __host__ __device__ static uint64_t* acc(void* base, int par, int src, int world, int rows,
                                             int D) {
        uint64_t* a0 = ml(base, 0, 0, world, rows) + size_t(2) * world * rows * 2;
        return a0 + (size_t)(par * world + src) * rows * D;
    }
};

// Waits (at most limit_ns) until the word at `addr` carries tag `epoch`;
// returns its value.  `ok` is cleared on timeout, after which no further
// waits are made.
__device__ __forceinline__ float x_wait_word(const uint64_t* addr, uint64_t w, uint32_t epoch,
                                             bool& ok, unsigned long long limit_ns) {
    if (uint32_t(w >> 32) != epoch && ok) {
        const unsigned long long t0 = globaltimer_ns();
        do {
            w = ld_relaxed_sys_u64(addr);
            if (uint32_t(w >> 32) == epoch) break;
            if (globaltimer_ns() - t0 > limit_ns) {
                ok = false;
                break;
            }
        } while (true);
    }
    return __uint_as_float(uint32_t(w));
}

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Named barrier over the consumer warps only (the producer may have exited).
__device__ __forceinline__ void consumer_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" :: "r"(nthreads) : "memory");
}

// Same barrier, returning the AND of `pred` over the participating threads.
__device__ __forceinline__ int consumer_sync_and(int pred, int nthreads) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"(pred), "r"(nthreads) : "memory");
    return r;
}

template <int D, int NT, int TILE, int STAGES, int NW>
struct SplitSmem {
    static constexpr int kSub = D / 64;                            // 128-byte column blocks
    static constexpr int kSubBytes = TILE * 128;                   // one [TILE][64] box
    static constexpr int kTileBytes = kSub * kSubBytes;            // K (or V) of one stage
    static constexpr size_t kRingBytes = size_t(2) * STAGES * kTileBytes;
    static constexpr size_t kBarOffset = kRingBytes;                // full, empty, recv
    // Cluster merge receive area (outside the ring: peers may push into it
    // while this CTA still streams): CL messages of [m GP][l GP][acc slice],
    // at most 2*GP*16 + GP*D floats for clusters of up to 16 CTAs.
    static constexpr size_t kRecvOffset =
        (kBarOffset + (2 * STAGES + 1) * sizeof(uint64_t) + 15) / 16 * 16;
    static constexpr size_t kRecvFloats = size_t(2 * NT * 8 * 16 + NT * 8 * D + 64);
    // +1024: the ring is realigned to 1024 bytes (128-byte swizzle atom).
    static constexpr size_t kBytes = 1024 + kRecvOffset + kRecvFloats * sizeof(float);
    // Cross-warp merge area (reuses the ring once every tile is consumed):
    // [NW][GP][kMergeStride] partial accumulators, rows padded by 4 floats so
    // the 4 lanes of a fragment column (heads 2t, 2t+2, ...) hit different
    // banks, then [NW][GP][2] (m, l) and [GP][NW] warp weights.
    static constexpr int kMergeStride = D + 4;
    static constexpr size_t kMergeBytes = size_t(NW) * (NT * 8) * kMergeStride * sizeof(float) +
                                          size_t(NW) * (NT * 8) * 3 * sizeof(float);
    // CTA state (acc [GP][D], m [GP], l [GP], flag) read by the cluster through DSMEM.
    static constexpr size_t kStateOffset = (kMergeBytes + 127) / 128 * 128;
    static constexpr size_t kStateBytes = size_t(NT * 8) * (D + 2) * sizeof(float) + 16;
    static_assert(kStateOffset + kStateBytes <= kRingBytes, "merge areas must fit in the ring");
    static_assert(kSubBytes % 1024 == 0, "swizzled boxes must stay 1024-byte aligned");
};

// Byte offset of the 16-byte chunk holding element (row r, column col) of a
// [rows][D] tile stored as D/64 swizzled [rows][64] boxes.
template <int TILE>
__device__ __forceinline__ uint32_t swz_offset(int r, int col) {
    const int sub = col >> 6;
    const int chunk = (col & 63) >> 3;
    return uint32_t(sub * TILE * 128 + r * 128 + ((chunk ^ (r & 7)) << 4));
}

// Cross-warp fold, one 8-head tile (nt) at a time: this lane's O^T
// fragments and its columns' (m, l) into / out of a row of the exchange area.
template <int D, int NT>
__device__ __forceinline__ void x_store(float* row, const float (&o)[D / 16][NT][4],
                                        const float (&m)[NT][2], const float (&l)[NT][2], int nt) {
#pragma unroll
    for (int dm = 0; dm < D / 16; ++dm)
        *reinterpret_cast<float4*>(row + dm * 4) =
            make_float4(o[dm][nt][0], o[dm][nt][1], o[dm][nt][2], o[dm][nt][3]);
    *reinterpret_cast<float4*>(row + (D / 16) * 4) =
        make_float4(m[nt][0], m[nt][1], l[nt][0], l[nt][1]);
}

template <int D, int NT>
__device__ __forceinline__ void x_fold(const float* row, float (&o)[D / 16][NT][4],
                                       float (&m)[NT][2], float (&l)[NT][2], int nt) {
    const float4 ml = *reinterpret_cast<const float4*>(row + (D / 16) * 4);
    const float mo[2] = {ml.x, ml.y}, lo[2] = {ml.z, ml.w};
    float sa[2], sb[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float mn = fmaxf(m[nt][j], mo[j]);
        const float mu = (mn == -INFINITY) ? 0.f : mn;
        sa[j] = fast_exp2(m[nt][j] - mu);
        sb[j] = fast_exp2(mo[j] - mu);
        l[nt][j] = fmaf(l[nt][j], sa[j], lo[j] * sb[j]);
        m[nt][j] = mn;
    }
#pragma unroll
    for (int dm = 0; dm < D / 16; ++dm) {
        const float4 v = *reinterpret_cast<const float4*>(row + dm * 4);
        o[dm][nt][0] = fmaf(o[dm][nt][0], sa[0], v.x * sb[0]);
        o[dm][nt][1] = fmaf(o[dm][nt][1], sa[1], v.y * sb[1]);
        o[dm][nt][2] = fmaf(o[dm][nt][2], sa[0], v.z * sb[0]);
        o[dm][nt][3] = fmaf(o[dm][nt][3], sa[1], v.w * sb[1]);
    }
}

// ---------------------------------------------------------------------------
// One consumer warp's share of one K/V tile: rows row0 .. row0 + 15 of the
// stage at kst / vst (shared-memory addresses; vgen = the V stage's generic
// address), of which the first valid_rows (>= 1) are real positions.
//   S^T = K Q^T (16 positions x GP heads), masked past valid_rows;
//   online softmax per head column in base 2 (m_run, l_run: this lane's
//   running max and partial row sum; o: the warp's O^T fragments);
//   O^T += V^T P^T with P = P_hi + P_lo (two fp16 halves).
// zero_tail: rows past the end may hold non-finite data (another
// sequence's rows of a pool); they are zeroed in V so P = 0 multiplies
// finite values.
// ---------------------------------------------------------------------------
template <int D, int NT, int TILE>
__device__ __forceinline__ void consume_tile(uint32_t kst, uint32_t vst, unsigned char* vgen,
                                             int row0, int valid_rows, bool zero_tail,
                                             const uint32_t (&qb)[D / 16][NT][2],
                                             float (&o)[D / 16][NT][4], float (&m_run)[NT][2],
                                             float (&l_run)[NT][2], float sl2, int lane) {
    constexpr int KSTEPS = D / 16;
    constexpr int DTILES = D / 16;
    constexpr int kSub = D / 64;
    constexpr int kSubBytes = TILE * 128;
    const int g = lane >> 2;
    // ldmatrix rows/columns of this lane (see the fragment maps in the file header).
    const int k_row = row0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int k_col = (lane >> 4) * 8;
    const int v_row = row0 + (lane & 7) + ((lane >> 4) & 1) * 8;
    const int v_col = ((lane >> 3) & 1) * 8;
    bool fenced = false;
    if (zero_tail && valid_rows < 16) {
        for (int c = lane; c < (16 - valid_rows) * kSub * 8; c += 32) {
            const int r = row0 + valid_rows + c / (kSub * 8);
            const int rest = c % (kSub * 8);
            *reinterpret_cast<uint4*>(vgen + (rest >> 3) * kSubBytes + r * 128 + (rest & 7) * 16) =
                make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
        fenced = true;
    }

    // ---- S^T = K Q^T (16 positions x GP heads)
    float sacc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) sacc[nt][c] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a0, a1, a2, a3, kst + swz_offset<TILE>(k_row, ks * 16 + k_col));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            mma_16816(sacc[nt], a0, a1, a2, a3, qb[ks][nt][0], qb[ks][nt][1]);
    }

    // ---- mask rows past the end
    const bool row_lo_ok = g < valid_rows;
    const bool row_hi_ok = g + 8 < valid_rows;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        if (!row_lo_ok) { sacc[nt][0] = -INFINITY; sacc[nt][1] = -INFINITY; }
        if (!row_hi_ok) { sacc[nt][2] = -INFINITY; sacc[nt][3] = -INFINITY; }
    }

    // ---- online softmax per head column (base 2)
    uint32_t pb[NT][2];
    uint32_t pl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float alpha[2];
        float pr[4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float mx = fmaxf(sacc[nt][j], sacc[nt][j + 2]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float m_new = fmaxf(m_run[nt][j], mx * sl2);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            alpha[j] = fast_exp2(m_run[nt][j] - m_use);
            m_run[nt][j] = m_new;
            pr[j] = fast_exp2(fmaf(sacc[nt][j], sl2, -m_use));
            pr[j + 2] = fast_exp2(fmaf(sacc[nt][j + 2], sl2, -m_use));
            l_run[nt][j] = fmaf(l_run[nt][j], alpha[j], pr[j] + pr[j + 2]);
        }
#pragma unroll
        for (int dm = 0; dm < DTILES; ++dm) {
            o[dm][nt][0] *= alpha[0];
            o[dm][nt][1] *= alpha[1];
            o[dm][nt][2] *= alpha[0];
            o[dm][nt][3] *= alpha[1];
        }
        // P^T fragments: rows = positions, cols = heads -> B layout
        // (k = pos, n = head).  P = P_hi + P_lo, both fp16.
        const __half2 h01 = __floats2half2_rn(pr[0], pr[1]);
        const __half2 h23 = __floats2half2_rn(pr[2], pr[3]);
        pb[nt][0] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&h01));
        pb[nt][1] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&h23));
        const float2 f01 = __half22float2(h01);
        const float2 f23 = __half22float2(h23);
        pl[nt][0] = movmatrix_trans(pack_half2(pr[0] - f01.x, pr[1] - f01.y));
        pl[nt][1] = movmatrix_trans(pack_half2(pr[2] - f23.x, pr[3] - f23.y));
    }

    // ---- O^T += V^T P^T
#pragma unroll
    for (int dm = 0; dm < DTILES; ++dm) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(a0, a1, a2, a3, vst + swz_offset<TILE>(v_row, dm * 16 + v_col));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            mma_16816(o[dm][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
            mma_16816(o[dm][nt], a0, a1, a2, a3, pl[nt][0], pl[nt][1]);
        }
    }
    // Generic-proxy writes into a stage the TMA will refill later.
    if (fenced) fence_proxy_async_smem();
}

// ---------------------------------------------------------------------------
// Split-KV decode kernel.
//   grid  = (Hkv * head_groups, num_splits, B), clusters of CL CTAs along y
//   block = 32 * (NW + 1): NW consumer warps + 1 producer warp (NW = 8 with
//   TILE = 64: two groups of four warps taking alternate tiles)
//
// Output paths (chosen by the host, uniform over the grid):
//   write_final        one split: the CTA writes fp16 out directly;
//   counters == null   unfused: each CTA writes its partial state to slot
//                      `split`; lse_merge_kernel runs next;
//   counters != null   fused: the CL CTAs of a cluster merge their states
//                      through distributed shared memory; with one cluster
//                      per (b, kv head, head group) that is the output,
//                      otherwise each cluster writes one partial and the last
//                      cluster to finish (atomic counter) merges them.
// With out_ml/out_acc set, the final result is a merged (m, l, acc) state
// instead of fp16 (used when KV ranges are split across GPUs).
//
// Launch overlap: the kernel lets the next grid launch at once
// (griddepcontrol.launch_dependents) and waits for the preceding grid
// (griddepcontrol.wait) before it reads q or writes anything; K/V tiles of
// rows below prefetch_rows may stream in before that wait.
// ---------------------------------------------------------------------------
// Launch bounds: the four-warp form leaves the register budget to the
// compiler (its choice, 94-162 registers by instantiation, is what was
// tuned); the eight-warp form runs one CTA per SM and is told so - left to
// itself the compiler aimed at three CTAs per SM and spilled.
template <int D, int NT, int TILE, int STAGES, int NW, int CL, bool PAGED>
__global__ void __launch_bounds__(32 * (NW + 1), NW > 4 ? 1 : 0)
split_decode_kernel(const __grid_constant__ DecodeParams p) {
    static_assert(D % 64 == 0, "head_dim must be a multiple of 64");
    // Consumer groups: NW warps of 16 rows each cover GR tiles at a time;
    // with GR = 2 the two groups of NW/2 warps take alternate tiles (group g
    // tiles g, g + 2, ...), so each group owns the stages s = g mod 2 of the
    // ring and never waits on a stage the other group consumes.
    constexpr int GR = 16 * NW / TILE;
    constexpr int WPG = NW / GR;                     // warps per group
    static_assert(GR * TILE == 16 * NW && (GR == 1 || GR == 2) && STAGES % GR == 0,
                  "each consumer warp owns one 16-row m-tile of its group's tiles");
    static_assert(CL >= 1 && CL <= 16, "cluster size");
    using S = SplitSmem<D, NT, TILE, STAGES, NW>;
    constexpr int GP = NT * 8;          // padded heads per CTA
    constexpr int KSTEPS = D / 16;      // k-steps of the QK product
    constexpr int DTILES = D / 16;      // m-tiles of the PV product

    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char* kring = smem;
    unsigned char* vring = smem + STAGES * S::kTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* recv_bar = empty + STAGES;                                 // cluster merge pushes
    float* recv = reinterpret_cast<float*>(smem + S::kRecvOffset);
    float* st_acc = reinterpret_cast<float*>(smem + S::kStateOffset);   // [GP][D]
    float* st_m = st_acc + GP * D;                                       // [GP]
    float* st_l = st_m + GP;                                             // [GP]
    uint32_t* st_flag = reinterpret_cast<uint32_t*>(st_l + GP);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // x = (kv head, head group): the CTAs that read the same cache rows of
    // one split launch back to back and stream those rows together.
    const int split = blockIdx.y;
    const int kvh = blockIdx.x / p.head_groups;
    const int hgrp = blockIdx.x % p.head_groups;
    const int b = blockIdx.z;

    // Heads served by this CTA: h0 .. h0 + gcount - 1.
    const int h0 = kvh * p.G + hgrp * GP;
    const int gcount = min(GP, p.G - hgrp * GP);

    // Sequence geometry.  A batch's lengths and row offsets may come from the
    // preceding kernel: read them after its completion unless the caller
    // declared them stable (prefetch_meta, launch overlap).
    if (p.kv_lens && !p.prefetch_meta) grid_dependency_wait();
    const int seq_len = p.kv_lens ? p.kv_lens[b] : p.kv_len;
    const long long row_base = p.row_offsets ? p.row_offsets[b] : 0;
    const int pos_begin = split * p.split_len;
    const int pos_end = min(seq_len, pos_begin + p.split_len);
    const int ntiles = pos_end > pos_begin ? (pos_end - pos_begin + TILE - 1) / TILE : 0;

    // Every CTA of this grid is running: the next grid may start launching.
    grid_launch_dependents();
    if (threadIdx.x == 0) FR_TRACE_EV(kEvStart);

    // Fused merge across a cluster: every CTA pushes each peer its (m, l) and
    // that peer's slice of acc (st.async into the peer's receive area, bytes
    // counted on the peer's recv_bar), so the merge needs no barrier after
    // the loop; the cluster barrier armed here only guarantees that every
    // CTA's recv_bar is initialised before anyone pushes.
    const bool cluster_merge = CL > 1 && p.counters != nullptr;
    const int x_nel = gcount * D;                    // merged elements of this unit
    const int x_per = (x_nel + CL - 1) / CL;         // slice per cluster rank (a multiple of 4)
    const int x_msg = 2 * GP + x_per;                // floats per message
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], WPG);               // one group consumes each stage
        }
        mbar_init(recv_bar, 1);
        if (cluster_merge) mbar_arrive_expect_tx(recv_bar, uint32_t(CL * x_msg * 4));
        fence_mbar_init();
    }
    __syncthreads();
    if (cluster_merge) cluster_arrive_release();

    bool ok = true;
    const int g = lane >> 2;     // fragment row group
    const int t = lane & 3;      // fragment column pair
    float o[DTILES][NT][4];
    float m_run[NT][2], l_run[NT][2];
    uint32_t xe_loaded = 0;          // exchange header (calls completed), read after the wait

    if (PAGED && warp == NW) {
        // -------------------------------------------------- paged producer
        // The whole warp walks the tiles.  Block-table entries are held 32 per
        // coalesced load (lane j: entry win + j; the next 32 already in
        // flight); lane j < TILE / page_box issues the copies of box j of the
        // tile, so one pass of the warp covers a tile whatever the page size.
        // Boxes past the end of the sequence, and page ids outside the pool,
        // read as zeros (a row coordinate past the tensor map).
        if (ntiles > 0) {
            if (lane == 0) {
                prefetch_tensormap(&p.kmap);
                prefetch_tensormap(&p.vmap);
            }
            const uint64_t policy = p.evict_normal ? l2_policy_evict_normal() : l2_policy_evict_first();
            grid_dependency_wait();                 // the block table may be the preceding grid's output
            const int* bt = p.block_table + (size_t)b * p.bt_stride;
            const int nent = min(p.bt_stride, (seq_len + p.page_size - 1) / p.page_size);
            const int box = p.page_box;
            const bool boxer = lane < TILE / box;
            const int oob_row = p.num_pages * p.page_size;
            int win = pos_begin / p.page_size;
            int mine = (win + lane < nent) ? __ldg(bt + win + lane) : -1;
            int ahead = (win + 32 + lane < nent) ? __ldg(bt + win + 32 + lane) : -1;
            int issued = 0;
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES) {
                    const bool w = mbar_wait_bounded(&empty[s], ((i / STAGES) - 1) & 1);
                    if (!__all_sync(0xffffffffu, w)) {
                        if (lane == 0) record_error(p.err, kDevTimeoutEmpty);
                        break;
                    }
                }
                const int t0 = pos_begin + i * TILE;
                // A tile spans at most TILE / 16 entries, so they lie in
                // [win, win + 64) once the window has moved past its first one.
                if (t0 / p.page_size >= win + 32) {
                    win += 32;
                    mine = ahead;
                    ahead = (win + 32 + lane < nent) ? __ldg(bt + win + 32 + lane) : -1;
                }
                const int tpos = t0 + lane * box;
                const int e = tpos / p.page_size;
                const int k = e - win;
                const int from_mine = __shfl_sync(0xffffffffu, mine, k & 31);
                const int from_ahead = __shfl_sync(0xffffffffu, ahead, k & 31);
                const int page = k < 32 ? from_mine : from_ahead;
                if (lane == 0) mbar_arrive_expect_tx(&full[s], uint32_t(2 * S::kTileBytes));
                __syncwarp();
                if (boxer) {
                    const int row = (tpos < seq_len && page >= 0 && page < p.num_pages)
                                        ? page * p.page_size + (tpos - e * p.page_size)
                                        : oob_row;
#pragma unroll
                    for (int sub = 0; sub < S::kSub; ++sub) {
                        const int o = s * S::kTileBytes + sub * S::kSubBytes + lane * box * 128;
                        tma_load_4d(kring + o, &p.kmap, 0, sub, kvh, row, &full[s], policy);
                        tma_load_4d(vring + o, &p.vmap, 0, sub, kvh, row, &full[s], policy);
                    }
                }
                ++issued;
            }
            // Drain (as below): no copy may still be in flight at exit.
            if (lane == 0) {
                for (int i = max(0, issued - STAGES); i < issued; ++i) {
                    if (!mbar_wait_bounded(&full[i % STAGES], (i / STAGES) & 1)) {
                        record_error(p.err, kDevTimeoutFull);
                        break;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == NW) {
        // -------------------------------------------------------- producer
        if (lane == 0 && ntiles > 0) {
            prefetch_tensormap(&p.kmap);
            prefetch_tensormap(&p.vmap);
            const uint64_t policy = p.evict_normal ? l2_policy_evict_normal() : l2_policy_evict_first();
            bool waited = false;
            int issued = 0;
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES) {
                    if (!mbar_wait_bounded(&empty[s], ((i / STAGES) - 1) & 1)) {
                        record_error(p.err, kDevTimeoutEmpty);
                        break;
                    }
                }
                const int t0 = pos_begin + i * TILE;
                if (!waited && t0 + TILE > p.prefetch_rows) {
                    grid_dependency_wait();
                    waited = true;
                }
                const int row = int(row_base + t0);
                mbar_arrive_expect_tx(&full[s], uint32_t(2 * S::kTileBytes));
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub) {
                    tma_load_4d(kring + s * S::kTileBytes + sub * S::kSubBytes, &p.kmap, 0, sub,
                                kvh, row, &full[s], policy);
                    tma_load_4d(vring + s * S::kTileBytes + sub * S::kSubBytes, &p.vmap, 0, sub,
                                kvh, row, &full[s], policy);
                }
                if (i == 0) FR_TRACE_EV(kEvFirstIssue);
                ++issued;
            }
            // Drain: wait until every copy this CTA issued has landed, so no
            // TMA write is still in flight when the ring is reused or the CTA
            // retires.
            for (int i = max(0, issued - STAGES); i < issued; ++i) {
                if (!mbar_wait_bounded(&full[i % STAGES], (i / STAGES) & 1)) {
                    record_error(p.err, kDevTimeoutFull);
                    break;
                }
            }
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------- consumers
        // q (and everything this CTA writes) depends on the preceding grid:
        // only an L2 prefetch of its lines may go before the wait (L2 stays
        // coherent, so a line the preceding kernel then writes is updated).
        if (warp == 0 && lane < (gcount * D * 2 + 127) / 128)
            prefetch_l2(p.q + ((size_t)b * p.H + h0) * D + lane * 64);
        grid_dependency_wait();
        // The exchange epoch: every call's last CTA advances it before the
        // grid ends, so it is final here; read now, used at the merge.
        if (p.xworld > 0 && threadIdx.x == 0) xe_loaded = __ldcg(XLayout::header(p.xbuf[p.xrank]));
        if (threadIdx.x == 0) FR_TRACE_EV(kEvDepWait);

        // Q^T as the B operand of S^T = K Q^T: b0 = Q[head][ks*16 + 2t .. +1], b1 = +8.
        uint32_t qb[KSTEPS][NT][2];
        {
            const __half* qrow_base = p.q + ((size_t)b * p.H + h0) * D;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int hj = nt * 8 + g;
                const bool valid = hj < gcount;
                const __half* qrow = qrow_base + (size_t)hj * D;
#pragma unroll
                for (int ks = 0; ks < KSTEPS; ++ks) {
                    qb[ks][nt][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t) : 0u;
                    qb[ks][nt][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t) : 0u;
                }
            }
        }

        if (threadIdx.x == 0) FR_TRACE_EV(kEvQLoaded);
#pragma unroll
        for (int dm = 0; dm < DTILES; ++dm)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int c = 0; c < 4; ++c) o[dm][nt][c] = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m_run[nt][0] = m_run[nt][1] = -INFINITY;
            l_run[nt][0] = l_run[nt][1] = 0.f;
        }

        const float sl2 = p.scale_log2;
        const int grp = warp / WPG;          // this warp's group: tiles grp, grp + GR, ...
        const int row0 = (warp - grp * WPG) * 16;   // its 16 rows of each of those tiles
        const uint32_t kring_s = smem_u32(kring);
        const uint32_t vring_s = smem_u32(vring);

        for (int i = grp; i < ntiles; i += GR) {
            const int s = i % STAGES;
            if (!mbar_wait_bounded(&full[s], (i / STAGES) & 1)) {
                record_error(p.err, kDevTimeoutFull);
                ok = false;
                break;
            }
            if (i == 0 && threadIdx.x == 0) FR_TRACE_EV(kEvFirstFull);
            const int tpos0 = pos_begin + i * TILE + row0;     // first position of this warp's m-tile
            if (tpos0 < pos_end)
                consume_tile<D, NT, TILE>(kring_s + s * S::kTileBytes, vring_s + s * S::kTileBytes,
                                          vring + s * S::kTileBytes, row0, pos_end - tpos0,
                                          p.zero_tail != 0, qb, o, m_run, l_run, sl2, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // Row sums: each lane summed its own positions; fold the 8 row groups.
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float l = l_run[nt][j];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                l_run[nt][j] = l;
            }

        if (threadIdx.x == 0) FR_TRACE_EV(kEvLoopEnd);
        // Every consumer must be past its last ldmatrix before the ring is
        // reused as the merge area.
        const int ok_all = consumer_sync_and(ok ? 1 : 0, NW * 32);
        if (threadIdx.x == 0) FR_TRACE_EV(kEvFoldSynced);

        // ---- cross-warp merge through shared memory -> CTA state
        constexpr int MS = S::kMergeStride;
        float* macc = reinterpret_cast<float*>(smem);                 // [NW][GP][MS]
        float* mml = macc + NW * GP * MS;                             // [NW][GP][2]
        float* wsc = mml + NW * GP * 2;                               // [GP][NW] warp weights
        if (ok_all) {
#pragma unroll
            for (int dm = 0; dm < DTILES; ++dm)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int d = dm * 16 + g + ((c >> 1) << 3);
                        const int hj = nt * 8 + 2 * t + (c & 1);
                        macc[(warp * GP + hj) * MS + d] = o[dm][nt][c];
                    }
            if (g == 0) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int hj = nt * 8 + 2 * t + j;
                        mml[(warp * GP + hj) * 2 + 0] = m_run[nt][j];
                        mml[(warp * GP + hj) * 2 + 1] = l_run[nt][j];
                    }
            }
        }
        if (threadIdx.x == 0) FR_TRACE_EV(kEvFoldStored);
        consumer_sync(NW * 32);
        // One thread per (head, warp), NW adjacent lanes per head: the max
        // over warps and the weighted l by shuffles, each warp's weight.
        static_assert((GP * NW) % 32 == 0 && 32 % NW == 0, "whole warps, heads within a warp");
        if (threadIdx.x < GP * NW) {
            const int hj = threadIdx.x / NW;
            const int w = threadIdx.x % NW;
            const float mw = ok_all ? mml[(w * GP + hj) * 2] : -INFINITY;
            const float lw = ok_all ? mml[(w * GP + hj) * 2 + 1] : 0.f;
            float mstar = mw;
#pragma unroll
            for (int o = 1; o < NW; o <<= 1) mstar = fmaxf(mstar, __shfl_xor_sync(0xffffffffu, mstar, o));
            const float muse = (mstar == -INFINITY) ? 0.f : mstar;
            const float sc = ok_all ? fast_exp2(mw - muse) : 0.f;
            wsc[hj * NW + w] = sc;
            float l = lw * sc;
#pragma unroll
            for (int o = 1; o < NW; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (w == 0) {
                st_m[hj] = mstar;
                st_l[hj] = l;
            }
        }
        consumer_sync(NW * 32);
        if (threadIdx.x == 0) FR_TRACE_EV(kEvFoldWeights);

        const size_t head_base = (size_t)b * p.H + h0;
        constexpr int kPerThread = GP * D / (NW * 32);
#pragma unroll
        for (int it = 0; it < kPerThread; ++it) {
            const int idx = threadIdx.x + it * NW * 32;
            const int hj = idx / D;
            const int d = idx % D;
            // A CTA whose bounded wait ran out (ok_all == 0, error word set)
            // carries the neutral state (m = -inf, l = 0, acc = 0) into every
            // merge, so no merge folds in the merge area's stale contents or a
            // partial slot left behind by an earlier call.
            float acc = 0.f;
            if (ok_all) {
#pragma unroll
                for (int w = 0; w < NW; ++w) acc = fmaf(macc[(w * GP + hj) * MS + d], wsc[hj * NW + w], acc);
            }
            const size_t hrow = head_base + hj;
            if (p.counters) {
                st_acc[hj * D + d] = acc;                    // fused: keep the CTA state
            } else if (hj < gcount) {
                const float l = st_l[hj];
                if (p.write_final) {
                    if (ok_all) p.out[hrow * D + d] = __float2half_rn(l > 0.f ? acc / l : 0.f);
                } else {
                    const size_t slot = hrow * p.part_slots + split;
                    p.part_acc[slot * D + d] = acc;
                    if (d == 0) {
                        p.part_ml[slot * 2 + 0] = st_m[hj];
                        p.part_ml[slot * 2 + 1] = l;
                    }
                }
            }
        }
    }

    if (threadIdx.x == 0) FR_TRACE_EV(kEvFold);
    if (!p.counters) return;       // unfused / single-split paths end here (uniform)
    if (threadIdx.x == 0) {
        st_flag[1] = xe_loaded;    // (the ring is free once every tile is consumed)
        // Exchange: count this CTA as having read the epoch (the release
        // orders the read before the count); the first CTA advances the
        // epoch for the next call once every CTA is counted.
        if (p.xworld > 0)
            red_add_release_gpu(reinterpret_cast<int*>(XLayout::header(p.xbuf[p.xrank]) + 1), 1);
    }
    __syncthreads();               // CTA state complete (producer included)
    if (threadIdx.x == 0) FR_TRACE_EV(kEvStateDone);

    // ------------------------------------------------------ fused merge
    // Level 1: the CL CTAs of the cluster merge their states through DSMEM;
    // CTA rank r merges element slice r of the (gcount x D) output.
    // Level 2 (several clusters per unit): slice r of every cluster partial is
    // written only by rank r, so the last rank-r CTA to finish (one counter
    // per (unit, rank)) merges slice r on its own - no second cluster barrier.
    const int crank = CL > 1 ? int(cluster_ctarank()) : 0;
    const int ncl = p.part_slots;                    // clusters per (b, kv head, head group)
    const int cl_id = split / CL;
    const size_t head_base = (size_t)b * p.H + h0;
    const int unit = (b * p.Hkv + kvh) * p.head_groups + hgrp;
    const int nel = gcount * D;
    const int per = (nel + CL - 1) / CL;
    const int e_begin = crank * per;
    const int e_end = min(nel, e_begin + per);
    const bool state_out = p.out_ml != nullptr;
    // Cross-GPU exchange: this call's epoch (the header advances only after
    // every CTA of the grid has finished) selects the buffer parity.
    const bool xmode = p.xworld > 0;
    const uint32_t xepoch = xmode ? st_flag[1] + 1u : 0u;
    const int xpar = int(xepoch & 1u);
    // Stores one element of a final state into every rank's exchange buffer
    // (tagged words, see XLayout).
    auto x_push = [&](size_t hrow, int d, float m, float l, float a) {
        const uint64_t tag = uint64_t(xepoch) << 32;
        for (int j = 0; j < p.xworld; ++j) {
            void* base = p.xbuf[j];
            st_relaxed_sys_u64(XLayout::acc(base, xpar, p.xrank, p.xworld, p.xrows, D) + hrow * D + d,
                               tag | __float_as_uint(a));
            if (d == 0) {
                uint64_t* mlp = XLayout::ml(base, xpar, p.xrank, p.xworld, p.xrows) + 2 * hrow;
                st_relaxed_sys_u64(mlp, tag | __float_as_uint(m));
                st_relaxed_sys_u64(mlp + 1, tag | __float_as_uint(l));
            }
        }
    };

    if constexpr (CL > 1) {
        // Push: message [m GP][l GP][acc slice j] to every cluster rank j,
        // stored at [my rank] of its receive area.
        cluster_wait_acquire();                      // every recv_bar is initialised
        if (threadIdx.x == 0) FR_TRACE_EV(kEvClusterReady);
        const int chunks = x_msg / 4;
        const uint32_t recv_s = smem_u32(recv), bar_s = smem_u32(recv_bar);
        for (int idx = threadIdx.x; idx < CL * chunks; idx += blockDim.x) {
            const int j = idx / chunks;
            const int f = (idx - j * chunks) * 4;    // first float of the chunk in the message
            float4 v;
            if (f < GP) {
                v = *reinterpret_cast<const float4*>(st_m + f);
            } else if (f < 2 * GP) {
                v = *reinterpret_cast<const float4*>(st_l + (f - GP));
            } else {
                const int e = j * x_per + (f - 2 * GP);
                v = e < x_nel ? *reinterpret_cast<const float4*>(st_acc + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            st_async_v4(dsmem_addr(recv_s + uint32_t(crank * x_msg + f) * 4u, uint32_t(j)), v,
                        dsmem_addr(bar_s, uint32_t(j)));
        }
        if (!mbar_wait_bounded(recv_bar, 0)) record_error(p.err, kDevTimeoutFull);
        if (threadIdx.x == 0) FR_TRACE_EV(kEvRecvDone);
    }
    {
        for (int e = e_begin + threadIdx.x; e < e_end; e += blockDim.x) {
            const int hj = e / D;
            const int d = e - hj * D;
            float mj[CL], lj[CL], aj[CL];
#pragma unroll
            for (int j = 0; j < CL; ++j) {
                if constexpr (CL > 1) {
                    const float* msg = recv + j * x_msg;
                    mj[j] = msg[hj];
                    lj[j] = msg[GP + hj];
                    aj[j] = msg[2 * GP + (e - e_begin)];
                } else {
                    mj[j] = st_m[hj];
                    lj[j] = st_l[hj];
                    aj[j] = st_acc[hj * D + d];
                }
            }
            float mstar = -INFINITY;
#pragma unroll
            for (int j = 0; j < CL; ++j) mstar = fmaxf(mstar, mj[j]);
            const float muse = (mstar == -INFINITY) ? 0.f : mstar;
            float a = 0.f, l = 0.f;
#pragma unroll
            for (int j = 0; j < CL; ++j) {
                const float sc = fast_exp2(mj[j] - muse);
                a = fmaf(aj[j], sc, a);
                l = fmaf(lj[j], sc, l);
            }
            const size_t hrow = head_base + hj;
            if (ncl == 1) {
                if (xmode) {
                    x_push(hrow, d, mstar, l, a);
                } else if (state_out) {
                    p.out_acc[hrow * D + d] = a;
                    if (d == 0) { p.out_ml[2 * hrow] = mstar; p.out_ml[2 * hrow + 1] = l; }
                } else {
                    p.out[hrow * D + d] = __float2half_rn(l > 0.f ? a / l : 0.f);
                }
            } else {
                const size_t slot = hrow * ncl + cl_id;
                p.part_acc[slot * D + d] = a;
                if (d == 0) { p.part_ml[2 * slot] = mstar; p.part_ml[2 * slot + 1] = l; }
            }
        }
    }
    if (threadIdx.x == 0) FR_TRACE_EV(kEvMergeEnd);
    if (ncl > 1) {
        __syncthreads();                             // slice stores of this CTA are done
        if (threadIdx.x == 0) {
            // acq_rel: publishes this CTA's slice (ordered before by the
            // barrier) and, for the last arriver, acquires the other slices.
            const int old = atom_add_acq_rel_gpu(&p.counters[unit * CL + crank], 1);
            st_flag[0] = (old == ncl - 1) ? 1u : 0u;
        }
        __syncthreads();
        if (st_flag[0]) {
            // Last rank-`crank` CTA: merge slice `crank` of all ncl partials,
            // every load of a chunk in flight at once.
            for (int e = e_begin + threadIdx.x; e < e_end; e += blockDim.x) {
                const int hj = e / D;
                const int d = e - hj * D;
                const size_t hrow = head_base + hj;
                const float* mlp = p.part_ml + 2 * hrow * ncl;
                const float* accp = p.part_acc + hrow * ncl * D + d;
                float m = -INFINITY, l = 0.f, a = 0.f;
                for (int c0 = 0; c0 < ncl; c0 += 8) {
                    float mv[8], lv[8], av[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const bool in = c0 + u < ncl;
                        mv[u] = in ? __ldcg(mlp + 2 * (c0 + u)) : -INFINITY;
                        lv[u] = in ? __ldcg(mlp + 2 * (c0 + u) + 1) : 0.f;
                        av[u] = in ? __ldcg(accp + (size_t)(c0 + u) * D) : 0.f;
                    }
                    float cm = m;
#pragma unroll
                    for (int u = 0; u < 8; ++u) cm = fmaxf(cm, mv[u]);
                    const float mu = (cm == -INFINITY) ? 0.f : cm;
                    const float r = fast_exp2(m - mu);
                    a *= r;
                    l *= r;
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const float w = fast_exp2(mv[u] - mu);
                        a = fmaf(av[u], w, a);
                        l = fmaf(lv[u], w, l);
                    }
                    m = cm;
                }
                if (xmode) {
                    x_push(hrow, d, m, l, a);
                } else if (state_out) {
                    p.out_acc[hrow * D + d] = a;
                    if (d == 0) { p.out_ml[2 * hrow] = m; p.out_ml[2 * hrow + 1] = l; }
                } else {
                    p.out[hrow * D + d] = __float2half_rn(l > 0.f ? a / l : 0.f);
                }
            }
            if (threadIdx.x == 0) p.counters[unit * CL + crank] = 0;   // ready for the next call
            if (threadIdx.x == 0) FR_TRACE_EV(kEvXMergeEnd);
        }
    }

    // ------------------------------------------------ cross-GPU exchange
    // The CTAs that pushed a final slice wait until every rank's words for
    // their slice carry this call's tag in the local buffer (all loads of an
    // element issued first, then only late words are polled), and merge the
    // slice over the ranks.
    if (xmode && (ncl == 1 || st_flag[0])) {
        void* xb = p.xbuf[p.xrank];
        const unsigned long long xlimit = 1000000ull * (unsigned long long)p.xwait_ms;
        bool ok = true;
        for (int e = e_begin + threadIdx.x; e < e_end; e += blockDim.x) {
            const int hj = e / D;
            const int d = e - hj * D;
            const size_t hrow = head_base + hj;
            uint64_t wm[kMaxRanks], wl[kMaxRanks], wa[kMaxRanks];
#pragma unroll
            for (int j = 0; j < kMaxRanks; ++j) {
                if (j < p.xworld) {
                    const uint64_t* mlp = XLayout::ml(xb, xpar, j, p.xworld, p.xrows) + 2 * hrow;
                    wm[j] = ld_relaxed_sys_u64(mlp);
                    wl[j] = ld_relaxed_sys_u64(mlp + 1);
                    wa[j] = ld_relaxed_sys_u64(XLayout::acc(xb, xpar, j, p.xworld, p.xrows, D) +
                                               hrow * D + d);
                }
            }
            float m = -INFINITY, l = 0.f, a = 0.f;
#pragma unroll
            for (int j = 0; j < kMaxRanks; ++j) {
                if (j < p.xworld) {
                    const uint64_t* mlp = XLayout::ml(xb, xpar, j, p.xworld, p.xrows) + 2 * hrow;
                    const float mj = x_wait_word(mlp, wm[j], xepoch, ok, xlimit);
                    const float lj = x_wait_word(mlp + 1, wl[j], xepoch, ok, xlimit);
                    const float aj = x_wait_word(
                        XLayout::acc(xb, xpar, j, p.xworld, p.xrows, D) + hrow * D + d, wa[j],
                        xepoch, ok, xlimit);
                    const float mn = fmaxf(m, mj);
                    const float mu = (mn == -INFINITY) ? 0.f : mn;
                    const float c_old = fast_exp2(m - mu), c_new = fast_exp2(mj - mu);
                    a = fmaf(a, c_old, aj * c_new);
                    l = fmaf(l, c_old, lj * c_new);
                    m = mn;
                }
            }
            p.out[hrow * D + d] = __float2half_rn(l > 0.f ? a / l : 0.f);
        }
        if (!ok) record_error(p.err, kDevTimeoutPeer);
    }
    if (xmode && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
        // The first CTA advances the epoch once every CTA of the grid has read
        // it (all of them counted themselves right after their tiles; the grid
        // is co-resident, so the count completes); the next call reads it after
        // this grid has ended.  The other CTAs leave without waiting.
        uint32_t* hdr = XLayout::header(p.xbuf[p.xrank]);
        const int total = int(gridDim.x * gridDim.y * gridDim.z);
        int* cnt = reinterpret_cast<int*>(hdr + 1);
        if (ld_acquire_gpu(cnt) < total) {
            const unsigned long long t0 = globaltimer_ns();
            while (ld_acquire_gpu(cnt) < total) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    record_error(p.err, kDevTimeoutPeer);
                    break;
                }
            }
        }
        hdr[1] = 0u;
        hdr[0] = xepoch;
    }
}

// ---------------------------------------------------------------------------
// Log-sum-exp merge of partial states.
//   grid = rows (one CTA per output head row), block = 256 threads (8 warps).
//   State s of row r: (m, l) = ml[r*ml_rs + s*ml_ss + {0, 1}] (m in log2
//   units), acc = acc[r*acc_rs + s*acc_ss + d]  (strides in floats).
//   Warp w folds states w, w+8, ... with online rescaling; lane owns dims
//   lane + 32j.  The warps' (m, l, acc) are folded once more in shared memory.
//   mode 0: out[r*D + d] = fp16( sum_s acc_s 2^(m_s-m*) / sum_s l_s 2^(m_s-m*) )
//   mode 1: merged state (m*, l*, acc*) into out_ml[2r..] / out_acc[r*D..],
//           so a rank can hand one state per head to the cross-GPU exchange.
// A row whose states are all empty (l = 0) yields zeros.
// ---------------------------------------------------------------------------
struct MergeStrides {
    long long ml_rs, ml_ss, acc_rs, acc_ss;
};

constexpr int kMergeWarps = 8;

template <int D>
__global__ void __launch_bounds__(32 * kMergeWarps)
lse_merge_kernel(const float* __restrict__ ml, const float* __restrict__ acc, int num_states,
                 const MergeStrides st, __half* __restrict__ out, float* __restrict__ out_ml,
                 float* __restrict__ out_acc, int mode) {
    constexpr int VEC = D / 32;
    __shared__ float s_acc[kMergeWarps][D];
    __shared__ float s_m[kMergeWarps], s_l[kMergeWarps];
    grid_launch_dependents();
    grid_dependency_wait();          // the partial states come from the preceding grid
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const float* mlr = ml + (size_t)r * st.ml_rs;
    const float* accr = acc + (size_t)r * st.acc_rs;

    float m = -INFINITY, l = 0.f, a[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) a[j] = 0.f;
    for (int s = warp; s < num_states; s += kMergeWarps) {
        const float ms = mlr[(size_t)s * st.ml_ss];
        const float ls = mlr[(size_t)s * st.ml_ss + 1];
        float v[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[j] = accr[(size_t)s * st.acc_ss + lane + 32 * j];
        const float mn = fmaxf(m, ms);
        const float mu = (mn == -INFINITY) ? 0.f : mn;
        const float c_old = fast_exp2(m - mu), c_new = fast_exp2(ms - mu);
        l = fmaf(l, c_old, ls * c_new);
#pragma unroll
        for (int j = 0; j < VEC; ++j) a[j] = fmaf(a[j], c_old, v[j] * c_new);
        m = mn;
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) s_acc[warp][lane + 32 * j] = a[j];
    if (lane == 0) { s_m[warp] = m; s_l[warp] = l; }
    __syncthreads();
    if (threadIdx.x < D) {
        const int d = threadIdx.x;
        float mstar = -INFINITY;
#pragma unroll
        for (int w = 0; w < kMergeWarps; ++w) mstar = fmaxf(mstar, s_m[w]);
        const float muse = (mstar == -INFINITY) ? 0.f : mstar;
        float at = 0.f, lt = 0.f;
#pragma unroll
        for (int w = 0; w < kMergeWarps; ++w) {
            const float sc = fast_exp2(s_m[w] - muse);
            at = fmaf(s_acc[w][d], sc, at);
            lt = fmaf(s_l[w], sc, lt);
        }
        if (mode == 0) {
            out[(size_t)r * D + d] = __float2half_rn(lt > 0.f ? at / lt : 0.f);
        } else {
            out_acc[(size_t)r * D + d] = at;
            if (d == 0) {
                out_ml[2 * r] = mstar;
                out_ml[2 * r + 1] = lt;
            }
        }
    }
}

}  // namespace fr
