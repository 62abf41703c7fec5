// batched_kernels.cuh - persistent, load-balanced decode over a ragged batch.
//
// Serves fr_decode_attn_batched: B sequences of different lengths in one KV
// pool, every (sequence, kv head, head group) "unit" needing its own
// softmax.  (The reference decodes one sequence per call,
// kernels/attention_decode.cu:535-556; batching is this library's addition.)
//
// Work decomposition (cost-balanced stream-K over K/V tiles).  Every unit
// is cut into 64-row tiles (at least one, so a zero-length sequence still
// yields zeros).  Concatenating all units' tiles in (sequence, kv head, head
// group) order gives T tiles; each unit is also charged a fixed cost before
// its first tile (starting an item) and after its last (its merge), in tile
// times (CostMap).  The grid is persistent - as many CTAs as are co-resident,
// fewer when that would leave under min_tiles_per_cta tiles each - and CTA c
// takes the c-th equal share of the total cost: every CTA is busy for the
// same time whatever the length distribution and wherever unit boundaries
// fall, and no CTA is launched without work.  A CTA's range is a sequence of
// "items" (the tiles of one unit inside the range): items in the middle of
// the range cover a whole unit; only the first and the last item can be a
// piece of a unit that other CTAs share.
//
// Per item: the consumer warps keep the split kernel's per-warp online
// softmax (consume_tile, decode_kernels.cuh) and fold their four states
// through a small shared-memory exchange area in two rounds (warps 2,3 ->
// 0,1 -> 0).  Warp 0 then writes the normalised fp16 output (whole unit) or
// stores the piece's (m, l, acc) state in the CTA's partial slot (2c for
// its first item, 2c + 1 for its last); the pieces are counted on their
// units' counters after the range (a release atomic per piece).
// The contributor whose count completes a unit merges it after its own range
// (log-sum-exp merge of the pieces in contributor order - the result does
// not depend on who merges - and re-arm): no CTA ever waits for another.
// Meanwhile the producer warp keeps streaming the next item's tiles through
// the TMA ring: the ring never drains at item boundaries.
//
// Metadata: every CTA reads kv_lens (B <= kPersistMaxBatch) and forms the
// tile prefix in shared memory with a block-wide scan; row_offsets are read
// by the producer one sequence ahead.
//
// Launch overlap: the kernel lets the next grid launch at once.  With
// prefetch_meta set (fr_set_launch_overlap(1) on a non-default stream) it
// reads kv_lens / row_offsets and streams every tile but each unit's last
// before its grid-dependency wait; q, the tiles holding a sequence's newest
// row, and every store wait for the preceding grid.
#pragma once
#include "decode_kernels.cuh"

namespace fr {

constexpr int kPersistMaxBatch = 512;   // sequences whose lengths fit the shared-memory prefix

template <int D, int NT, int TILE, int STAGES, int NW>
struct PersistSmem {
    static constexpr int kSub = D / 64;
    static constexpr int kSubBytes = TILE * 128;
    static constexpr int kTileBytes = kSub * kSubBytes;
    static constexpr size_t kRingBytes = size_t(2) * STAGES * kTileBytes;
    // Exchange area of the cross-warp fold: 2 slots x 32 lanes x (the O^T
    // fragments of one 8-head tile + m, l of its two head columns).
    static constexpr int kXFloats = (D / 16) * 4 + 4;
    static constexpr size_t kXOffset = kRingBytes;
    static constexpr size_t kXBytes = size_t(2) * 32 * kXFloats * sizeof(float);
    static constexpr size_t kBarOffset = kXOffset + kXBytes;            // full, empty
    static constexpr size_t kFlagOffset = kBarOffset + 2 * STAGES * sizeof(uint64_t);
    static constexpr size_t kMetaOffset = kFlagOffset + 16 * sizeof(int);
    // seq_start [kPersistMaxBatch + 1] (tile prefix x units per sequence),
    // lens [kPersistMaxBatch], warp sums [8]
    static constexpr size_t kMetaBytes = (2 * kPersistMaxBatch + 1 + 8) * sizeof(int);
    // +1024: the ring is realigned to 1024 bytes (128-byte swizzle atom).
    static constexpr size_t kBytes = 1024 + kMetaOffset + kMetaBytes;
    static_assert(kSubBytes % 1024 == 0, "swizzled boxes must stay 1024-byte aligned");
    static_assert(kXFloats % 4 == 0, "exchange rows are float4-stored");
};

// Tiles per sequence (at least one) as an exclusive prefix in unit tiles
// (x upb units per sequence): seq_start[0..B]; lens[b] = kv_lens[b].  Every
// thread of the block takes part.
template <int TILE>
__device__ __forceinline__ void scan_lengths(const int* kv_lens, int B, int upb, int* seq_start,
                                             int* lens, int* warp_sums) {
    constexpr int kChunks = 4;                      // 4 x 160 threads >= kPersistMaxBatch
    const int nthr = blockDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = nthr >> 5;
    int vals[kChunks];
#pragma unroll
    for (int r = 0; r < kChunks; ++r) {             // every load in flight at once
        const int b = r * nthr + tid;
        vals[r] = b < B ? kv_lens[b] : 0;
    }
    int carry = 0;
#pragma unroll
    for (int r = 0; r < kChunks; ++r) {
        if (r * nthr >= B) break;                   // uniform
        const int b = r * nthr + tid;
        const int len = max(0, vals[r]);
        const int n = b < B ? max(1, (len + TILE - 1) / TILE) : 0;
        int x = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < nwarps; ++w) {
            const int ws = warp_sums[w];
            before += w < warp ? ws : 0;
            total += ws;
        }
        if (b < B) {
            seq_start[b] = (carry + before + x - n) * upb;
            lens[b] = len;
        }
        carry += total;
        __syncthreads();                            // warp_sums is reused
    }
    if (tid == 0) seq_start[B] = carry * upb;
    __syncthreads();                                // the prefix is complete for every thread
}

// Position in the concatenated tile list: sequence b, unit j within the
// sequence (kv head * head_groups + head group), tile i within the unit,
// nb = tiles per unit of sequence b.
struct TileCursor {
    int b, j, i, nb;
    __device__ __forceinline__ void seek(const int* seq_start, int B, int upb, int t) {
        int lo = 0, hi = B - 1;                     // last b with seq_start[b] <= t
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (seq_start[mid] <= t) lo = mid; else hi = mid - 1;
        }
        b = lo;
        nb = (seq_start[b + 1] - seq_start[b]) / upb;
        const int off = t - seq_start[b];
        j = off / nb;
        i = off - j * nb;
    }
    // Moves n tiles on, n <= nb - i (never past the end of the unit); past
    // the last sequence the cursor is left at b == B with nb = 1.
    __device__ __forceinline__ void advance(const int* seq_start, int B, int upb, int n) {
        i += n;
        if (i == nb) {
            i = 0;
            if (++j == upb) {
                j = 0;
                ++b;
                nb = b < B ? (seq_start[b + 1] - seq_start[b]) / upb : 1;
            }
        }
    }
};

// Cost-balanced partition.  Every unit costs its tiles plus `xc` tile-times
// placed before its first tile (starting an item: q load, and the fold and
// piece store of the item it ends) and `mc` after its last tile (a share of
// the merge cost, charged to the CTA holding that tile).  In cost space unit j of sequence b
// spans xc + nb + mc points from cs(b) + j * (nb + xc + mc), the sequence's
// cost start being cs(b) = seq_start[b] + (xc + mc) * upb * b.  CTA c owns
// the cost range [c*Ctot/C, (c+1)*Ctot/C);
// its tiles are those whose cost points fall in it (the unit's first tile
// also owns the xc points before it, its last tile the mc points after it).
// With Ctot / C >= xc + mc + 2 every CTA owns at least one tile.
struct CostMap {
    const int* seq_start;
    int B, upb, xc, mc;
    long long Ctot, C;

    __device__ __forceinline__ long long cs(int b) const {
        return seq_start[b] + (long long)(xc + mc) * upb * b;
    }
    // first tile whose cost points reach v (v < Ctot)
    __device__ __forceinline__ int tile_at(long long v) const {
        int lo = 0, hi = B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (cs(mid) <= v) lo = mid; else hi = mid - 1;
        }
        const int nb = (seq_start[lo + 1] - seq_start[lo]) / upb;
        const long long span = nb + xc + mc;
        const long long off = v - cs(lo);
        const int j = (int)min(off / span, (long long)(upb - 1));
        const long long r = off - j * span;
        const int i = (int)max(0LL, min(r - xc, (long long)(nb - 1)));
        return seq_start[lo] + j * nb + i;
    }
    __device__ __forceinline__ int beg(long long c) const {
        return c >= C ? seq_start[B] : tile_at((c * Ctot) / C);
    }
    // CTA owning the last cost point of tile i of unit j of sequence b
    __device__ __forceinline__ int cta_of(int b, int j, int nb, int i) const {
        const long long hi = cs(b) + (long long)j * (nb + xc + mc) + xc + i + (i == nb - 1 ? mc : 0);
        return int(((hi + 1) * C - 1) / Ctot);
    }
};

// Merges the pieces of a unit, stored by contributors cf..cl (CTA c's slot is
// 2c, or 2c + 1 for cf when the unit is not its first item), into the fp16
// output of the unit's gcount heads.  Pieces are kept in the consumer
// fragment order - slot [dm][nt][lane] float4 = o[dm][nt][0..3] of that
// lane, then (m, l) per head - so every thread folds whole float4
// fragments: fragment f = (dm, nt, lane) holds heads nt*8 + 2(lane&3) +
// {0,1} at dims dm*16 + lane/4 + {0,8}.
//
// Contributors go in chunks of KW = threads / GP.  Per chunk the first UB
// contributors' fragments are requested first; meanwhile thread (head h,
// contributor u) loads that piece's (m, l), the KW lanes of a head form the
// chunk's maximum and weighted row sum by shuffles, and the weights
// 2^(m_u - m) go to shared memory; after one barrier every thread folds its
// fragments with FMAs only.  The order of the sums is fixed (contributor
// order within a lane group, lanes by shuffle tree), so the result does not
// depend on which CTA merges.  All consumer threads take part.
template <int D, int NT, int NW>
__device__ __forceinline__ void merge_pieces(const DecodeParams& p, float* area, int cf, int cl,
                                             bool cf_tail, int gcount, size_t head_base) {
    constexpr int GP = NT * 8;
    constexpr int DTILES = D / 16;
    constexpr int NTHR = NW * 32;
    constexpr int KW = NTHR / GP;                         // contributors per chunk
    constexpr int NFRAG = DTILES * NT * 32;               // float4 fragments per piece
    constexpr int FPT = NFRAG / NTHR;                     // fragments per thread
    constexpr int UB = 16 / FPT;                          // contributors per load batch
    static_assert(NFRAG % NTHR == 0 && KW <= 32 && 32 % KW == 0, "merge thread layout");
    float* sm_w = area;                                   // [KW][GP] chunk weights
    float* sm_r = sm_w + KW * GP;                         // [GP] rescale of the running state
    float* sm_inv = sm_r + GP;                            // [GP] 1 / final row sum
    const int tid = threadIdx.x;
    const int wh = tid / KW, wu = tid - (tid / KW) * KW;  // weight thread: head, contributor
    float mrun = -INFINITY, lrun = 0.f;                   // head wh's running state (its KW lanes)
    float4 acc[FPT];
    int ha[FPT];                                          // first head of the fragment
#pragma unroll
    for (int i = 0; i < FPT; ++i) {
        acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int f = tid + i * NTHR;
        ha[i] = ((f >> 5) % NT) * 8 + 2 * (f & 3);
    }
    auto slot_of = [&](int cc) { return 2 * cc + ((cc == cf && cf_tail) ? 1 : 0); };
    const int k_all = cl - cf + 1;
    for (int c0 = 0; c0 < k_all; c0 += KW) {
        const int kc = min(KW, k_all - c0);
        float4 v[FPT][UB];
        auto load_batch = [&](int u0) {
#pragma unroll
            for (int i = 0; i < FPT; ++i)
#pragma unroll
                for (int u = 0; u < UB; ++u) {
                    const int f = tid + i * NTHR;
                    const float4* src = reinterpret_cast<const float4*>(
                        p.part_acc + (size_t)slot_of(cf + c0 + u0 + u) * GP * D) + f;
                    v[i][u] = u0 + u < kc ? __ldcg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
        };
        consumer_sync(NTHR);                              // the previous chunk's weights are used
        load_batch(0);                                    // in flight with the (m, l) loads
        float m = -INFINITY, l = 0.f;
        if (wu < kc) {
            const float* pm = p.part_ml + ((size_t)slot_of(cf + c0 + wu) * GP + wh) * 2;
            m = __ldcg(pm);
            l = __ldcg(pm + 1);
        }
        float mx = m;
#pragma unroll
        for (int o = 1; o < KW; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mnew = fmaxf(mrun, mx);
        const float muse = (mnew == -INFINITY) ? 0.f : mnew;
        const float w = fast_exp2(m - muse);              // 0 for an empty piece (m = -inf)
        const float r = fast_exp2(mrun - muse);
        float ls = l * w;
#pragma unroll
        for (int o = 1; o < KW; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        lrun = fmaf(lrun, r, ls);
        mrun = mnew;
        sm_w[wu * GP + wh] = w;
        if (wu == 0) {
            sm_r[wh] = r;
            sm_inv[wh] = lrun > 0.f ? 1.f / lrun : 0.f;
        }
        consumer_sync(NTHR);
        if (tid == 0) FR_TRACE_EV(kEvMergeLoaded);
#pragma unroll
        for (int i = 0; i < FPT; ++i) {
            const float r0 = sm_r[ha[i]], r1 = sm_r[ha[i] + 1];
            acc[i].x *= r0; acc[i].y *= r1; acc[i].z *= r0; acc[i].w *= r1;
        }
        for (int u0 = 0; u0 < kc; u0 += UB) {
            if (u0 > 0) load_batch(u0);
#pragma unroll
            for (int i = 0; i < FPT; ++i)
#pragma unroll
                for (int u = 0; u < UB; ++u) {
                    if (u0 + u < kc) {
                        const float w0 = sm_w[(u0 + u) * GP + ha[i]];
                        const float w1 = sm_w[(u0 + u) * GP + ha[i] + 1];
                        acc[i].x = fmaf(v[i][u].x, w0, acc[i].x);
                        acc[i].y = fmaf(v[i][u].y, w1, acc[i].y);
                        acc[i].z = fmaf(v[i][u].z, w0, acc[i].z);
                        acc[i].w = fmaf(v[i][u].w, w1, acc[i].w);
                    }
                }
        }
    }
#pragma unroll
    for (int i = 0; i < FPT; ++i) {
        const int f = tid + i * NTHR;
        const int d = (f / (32 * NT)) * 16 + ((f & 31) >> 2);
        const float vals[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int h = ha[i] + (c & 1);
            if (h < gcount)
                p.out[(head_base + h) * D + d + ((c >> 1) << 3)] = __float2half_rn(vals[c] * sm_inv[h]);
        }
    }
}

// ---------------------------------------------------------------------------
// Persistent batched decode kernel.
//   grid  = C CTAs (co-resident), block = 32 * (NW + 1): NW consumer warps +
//   one producer warp.  p.batch sequences, p.Hkv kv heads, p.head_groups
//   head groups of GP = 8 * NT query heads per kv head.
//   p.counters: one per unit, zero between calls; p.part_ml / p.part_acc:
//   2 * C partial slots of [GP][2] / [GP][D] floats.
// ---------------------------------------------------------------------------
template <int D, int NT, int TILE, int STAGES, int NW>
__global__ void __launch_bounds__(32 * (NW + 1), 2)
persistent_decode_kernel(const __grid_constant__ DecodeParams p) {
    static_assert(TILE == 16 * NW, "each consumer warp owns one 16-row m-tile per stage");
    using S = PersistSmem<D, NT, TILE, STAGES, NW>;
    constexpr int GP = NT * 8;
    constexpr int KSTEPS = D / 16;
    constexpr int DTILES = D / 16;
    constexpr int XF = S::kXFloats;

    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char* kring = smem;
    unsigned char* vring = smem + STAGES * S::kTileBytes;
    float* xarea = reinterpret_cast<float*>(smem + S::kXOffset);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + STAGES;
    int* xflag = reinterpret_cast<int*>(smem + S::kFlagOffset);
    int* seq_start = reinterpret_cast<int*>(smem + S::kMetaOffset);
    int* lens = seq_start + kPersistMaxBatch + 1;
    int* warp_sums = lens + kPersistMaxBatch;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int B = p.batch;
    const int hg = p.head_groups;
    const int upb = p.Hkv * hg;                     // units per sequence

    grid_launch_dependents();
    if (threadIdx.x == 0) FR_TRACE_EV(kEvStart);
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    if (!p.prefetch_meta) grid_dependency_wait();  // lengths may come from the preceding grid
    scan_lengths<TILE>(p.kv_lens, B, upb, seq_start, lens, warp_sums);  // ends in a barrier

    // C <= T CTAs take part, so every one of them owns at least one tile: the
    // CTAs whose ranges meet a unit are exactly the ones that store a piece
    // of it (the merge counts on that).
    // Few tiles per CTA: fewer CTAs, each with a longer range (its fixed
    // costs - first tile, fold, piece store - weigh less, and the freed SM
    // slots let the next launch's CTAs start early).
    const long long T = seq_start[B];
    CostMap cm{seq_start, B, upb, p.item_cost, p.merge_cost, 0, 0};
    cm.Ctot = T + (long long)B * upb * (cm.xc + cm.mc);
    long long C = min((long long)gridDim.x, T);
    if (p.min_tiles_per_cta > 0)
        C = min(C, max((long long)p.min_ctas, T / p.min_tiles_per_cta));
    C = max(1LL, min(C, cm.Ctot / (cm.xc + cm.mc + 2)));   // every CTA owns a tile
    cm.C = C;
    if (blockIdx.x >= C) return;                    // uniform over the CTA
    const int beg = cm.beg(blockIdx.x);
    const int end = cm.beg(blockIdx.x + 1);
    const int n = end - beg;
    if (threadIdx.x == 0) FR_TRACE_EV(kEvMeta);

    TileCursor start;
    start.seek(seq_start, B, upb, beg);

    if (warp == NW) {
        // -------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&p.kmap);
            prefetch_tensormap(&p.vmap);
            const uint64_t policy = p.evict_normal ? l2_policy_evict_normal() : l2_policy_evict_first();
            bool waited = !p.prefetch_meta;
            TileCursor cur = start;
            int cb = cur.b;
            long long rowb = p.row_offsets ? p.row_offsets[cb] : 0;
            long long rown = (p.row_offsets && cb + 1 < B) ? p.row_offsets[cb + 1] : 0;
            int issued = 0;
            for (int k = 0; k < n; ++k) {
                const int s = k % STAGES;
                if (k >= STAGES && !mbar_wait_bounded(&empty[s], ((k / STAGES) - 1) & 1)) {
                    record_error(p.err, kDevTimeoutEmpty);
                    break;
                }
                if (cur.b != cb) {                  // next sequence (b grows by one)
                    cb = cur.b;
                    rowb = rown;
                    rown = (p.row_offsets && cb + 1 < B) ? p.row_offsets[cb + 1] : 0;
                }
                // a unit's last tile holds its sequence's newest row
                if (!waited && cur.i == cur.nb - 1) {
                    grid_dependency_wait();
                    waited = true;
                }
                const int kvh = cur.j / hg;
                const int row = int(rowb + (long long)cur.i * TILE);
                mbar_arrive_expect_tx(&full[s], uint32_t(2 * S::kTileBytes));
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub) {
                    tma_load_4d(kring + s * S::kTileBytes + sub * S::kSubBytes, &p.kmap, 0, sub,
                                kvh, row, &full[s], policy);
                    tma_load_4d(vring + s * S::kTileBytes + sub * S::kSubBytes, &p.vmap, 0, sub,
                                kvh, row, &full[s], policy);
                }
                if (k == 0) FR_TRACE_EV(kEvFirstIssue);
                ++issued;
                cur.advance(seq_start, B, upb, 1);
            }
            // Drain: every copy this CTA issued has landed before it retires.
            for (int i = max(0, issued - STAGES); i < issued; ++i) {
                if (!mbar_wait_bounded(&full[i % STAGES], (i / STAGES) & 1)) {
                    record_error(p.err, kDevTimeoutFull);
                    break;
                }
            }
        }
        __syncwarp();
        return;
    }

    // ------------------------------------------------------------ consumers
    // Merge bookkeeping of the range's first and last item, worked out while
    // the preceding grid still runs (with launch overlap): xm[6r..6r+5] =
    // unit (-1: not shared with other CTAs), first and last contributor,
    // whether the unit is not the first contributor's first item, sequence,
    // unit index; r = 0 for the first item (slot 2c), 1 for the last (2c + 1).
    int* xm = xflag + 2;
    if (threadIdx.x == 0) {
        TileCursor lc;
        lc.seek(seq_start, B, upb, end - 1);
        const bool one = start.b == lc.b && start.j == lc.j;
        auto note = [&](int r, int bb, int jj, int nbb, bool shared) {
            int* m = xm + 6 * r;
            m[0] = shared ? bb * upb + jj : -1;
            if (!shared) return;
            m[1] = cm.cta_of(bb, jj, nbb, 0);
            m[2] = cm.cta_of(bb, jj, nbb, nbb - 1);
            m[3] = cm.beg(m[1]) < seq_start[bb] + jj * nbb ? 1 : 0;
            m[4] = bb;
            m[5] = jj;
        };
        note(0, start.b, start.j, start.nb,
             one ? !(start.i == 0 && lc.i == lc.nb - 1) : start.i != 0);
        note(1, lc.b, lc.j, lc.nb, !one && lc.i != lc.nb - 1);
    }
    if (p.prefetch_meta) {
        // q and the outputs depend on the preceding grid; only an L2 prefetch
        // of the first item's q lines may go before the wait (L2 stays
        // coherent, so a line the preceding kernel then writes is updated)
        const int kvh0 = start.j / hg, hg0 = start.j - kvh0 * hg;
        const int gc0 = min(GP, p.G - hg0 * GP);
        if (warp == 0 && lane < (gc0 * D * 2 + 127) / 128)
            prefetch_l2(p.q + ((size_t)start.b * p.H + kvh0 * p.G + hg0 * GP) * D + lane * 64);
        grid_dependency_wait();
    }
    if (threadIdx.x == 0) FR_TRACE_EV(kEvDepWait);
    const int g = lane >> 2;
    const int t = lane & 3;
    const int row0 = warp * 16;
    const float sl2 = p.scale_log2;
    const uint32_t kring_s = smem_u32(kring);
    const uint32_t vring_s = smem_u32(vring);
    bool ok = true;
    TileCursor cur = start;
    int k = 0;
    for (int e = 0; k < n; ++e) {
        const int b = cur.b, j = cur.j, nb = cur.nb, i0 = cur.i;
        const int cnt = min(nb - i0, n - k);
        const int kvh = j / hg, hgrp = j - (j / hg) * hg;
        const int h0 = kvh * p.G + hgrp * GP;
        const int gcount = min(GP, p.G - hgrp * GP);
        const int len = lens[b];
        const int ustart = seq_start[b] + j * nb;  // the unit's first tile in the list
        const size_t head_base = (size_t)b * p.H + h0;

        // Q^T as the B operand of S^T = K Q^T
        uint32_t qb[KSTEPS][NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int hj = nt * 8 + g;
            const bool valid = hj < gcount;
            const __half* qrow = p.q + (head_base + hj) * D;
#pragma unroll
            for (int ks = 0; ks < KSTEPS; ++ks) {
                qb[ks][nt][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t) : 0u;
                qb[ks][nt][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t) : 0u;
            }
        }
        if (threadIdx.x == 0) FR_TRACE_EV(kEvQLoaded);
        float o[DTILES][NT][4];
        float m_run[NT][2], l_run[NT][2];
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

        for (int tt = 0; tt < cnt; ++tt, ++k) {
            const int s = k % STAGES;
            // After a timed-out wait the warp stops reading the ring but keeps
            // walking the items, so every consumer barrier below still meets.
            if (ok && !mbar_wait_bounded(&full[s], (k / STAGES) & 1)) {
                record_error(p.err, kDevTimeoutFull);
                ok = false;
            }
            if (k == 0 && threadIdx.x == 0) FR_TRACE_EV(kEvFirstFull);
            const int tpos0 = (i0 + tt) * TILE + row0;
            if (ok && tpos0 < len)
                consume_tile<D, NT, TILE>(kring_s + s * S::kTileBytes, vring_s + s * S::kTileBytes,
                                          vring + s * S::kTileBytes, row0, len - tpos0,
                                          p.zero_tail != 0, qb, o, m_run, l_run, sl2, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        cur.advance(seq_start, B, upb, cnt);
        if (threadIdx.x == 0) FR_TRACE_EV(kEvLoopEnd);

        // Row sums: each lane summed its own positions; fold the 8 row groups.
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                float l = l_run[nt][jj];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                l_run[nt][jj] = l;
            }

        // ---- cross-warp fold: warps 2,3 -> 0,1, then 1 -> 0
        const int ok_all = consumer_sync_and(ok ? 1 : 0, NW * 32);
        static_assert(NW == 4, "two fold rounds");
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if (warp >= 2) x_store<D, NT>(xarea + ((warp - 2) * 32 + lane) * XF, o, m_run, l_run, nt);
            consumer_sync(NW * 32);
            if (warp < 2) x_fold<D, NT>(xarea + (warp * 32 + lane) * XF, o, m_run, l_run, nt);
            consumer_sync(NW * 32);
            if (warp == 1) x_store<D, NT>(xarea + lane * XF, o, m_run, l_run, nt);
            consumer_sync(NW * 32);
            if (warp == 0) x_fold<D, NT>(xarea + lane * XF, o, m_run, l_run, nt);
            consumer_sync(NW * 32);
        }

        if (threadIdx.x == 0) FR_TRACE_EV(kEvFold);
        // ---- output of the item
        const bool whole = i0 == 0 && cnt == nb;
        if (whole) {
            if (warp == 0 && ok_all) {
#pragma unroll
                for (int dm = 0; dm < DTILES; ++dm)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const int d = dm * 16 + g + ((c >> 1) << 3);
                            const int hj = nt * 8 + 2 * t + (c & 1);
                            const float l = l_run[nt][c & 1];
                            if (hj < gcount)
                                p.out[(head_base + hj) * D + d] =
                                    __float2half_rn(l > 0.f ? o[dm][nt][c] / l : 0.f);
                        }
            }
            if (threadIdx.x == 0) FR_TRACE_EV(kEvStored);
            continue;
        }
        // A piece of a unit shared with other CTAs, in fragment order
        // (merge_pieces), in slot 2c (first item of this CTA) or 2c + 1 (its
        // last); a timed-out CTA stores the neutral state (m = -inf, l = 0,
        // acc = 0).  The stores are not waited for here: under the full
        // K/V stream a fence takes microseconds, and a first item's fence
        // would stall the ring for the items behind it.  Pieces are counted
        // after the range.
        if (warp == 0) {
            const int slot = 2 * blockIdx.x + (e == 0 ? 0 : 1);
            float4* pa = reinterpret_cast<float4*>(p.part_acc + (size_t)slot * GP * D);
            float* pm = p.part_ml + (size_t)slot * GP * 2;
#pragma unroll
            for (int dm = 0; dm < DTILES; ++dm)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    pa[(dm * NT + nt) * 32 + lane] =
                        ok_all ? make_float4(o[dm][nt][0], o[dm][nt][1], o[dm][nt][2], o[dm][nt][3])
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            if (g == 0) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int jj = 0; jj < 2; ++jj) {
                        const int hj = nt * 8 + 2 * t + jj;
                        pm[hj * 2 + 0] = ok_all ? m_run[nt][jj] : -INFINITY;
                        pm[hj * 2 + 1] = ok_all ? l_run[nt][jj] : 0.f;
                    }
            }
        }
        if (threadIdx.x == 0) FR_TRACE_EV(kEvStored);
    }

    // ---- count the pieces, then merge every unit whose count this CTA
    // completed: all its pieces are stored and visible (each contributor
    // counts with release semantics - warp 0's stores are ordered before lane
    // 0's count by __syncwarp - and the merging CTA fences after reading the
    // count; its other threads follow through the barrier).
    // The merge reads the pieces in contributor order, so the result does not
    // depend on which contributor merges.
    if (warp == 0) {
        __syncwarp();
        if (lane == 0) {
            int f0 = 0, f1 = 0;
            if (xm[0] >= 0 || xm[6] >= 0) {
                // each count releases this CTA's pieces
                if (xm[0] >= 0) f0 = atom_add_release_gpu(&p.counters[xm[0]], 1) == xm[2] - xm[1];
                if (xm[6] >= 0) f1 = atom_add_release_gpu(&p.counters[xm[6]], 1) == xm[8] - xm[7];
                if (f0 | f1) fence_acq_rel_gpu();      // acquire the other contributors' pieces
            }
            xflag[0] = f0;
            xflag[1] = f1;
            FR_TRACE_EV(kEvCounted);
        }
    }
    consumer_sync(NW * 32);
#pragma unroll 1
    for (int r = 0; r < 2; ++r) {                      // flags are uniform over the consumer warps
        if (!xflag[r]) continue;
        const int* m = xm + 6 * r;
        const int bb = m[4], jj = m[5];
        const int kvh = jj / hg, hgrp = jj - (jj / hg) * hg;
        const int gcount = min(GP, p.G - hgrp * GP);
        const size_t head_base = (size_t)bb * p.H + kvh * p.G + hgrp * GP;
        if (threadIdx.x == 0) FR_TRACE_EV(kEvMergeBegin);
        merge_pieces<D, NT, NW>(p, xarea, m[1], m[2], m[3] != 0, gcount, head_base);
        if (threadIdx.x == 0) {
            p.counters[m[0]] = 0;                      // every piece was counted: re-arm
            FR_TRACE_EV(kEvMergeEnd);
        }
    }
}

}  // namespace fr
