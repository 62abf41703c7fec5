// capi.cu - extern "C" entry points of libforgert_b200.so.
//
// Argument checks, per-device state (SM count, error word, workspace), TMA
// tensor-map encoding, the split planner and the kernel launches.
// Declarations and contracts live in include/forgert_attn.h; each entry point
// there names the reference launcher it replaces.
#include "decode_kernels.cuh"
#include "batched_kernels.cuh"
#include "prefill_kernels.cuh"
#include "prefill_tc_kernels.cuh"
#include "rope_kernels.cuh"
#include "copy_kernels.cuh"
#include "../../include/forgert_attn.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <numeric>
#include <vector>

namespace {

using fr::DecodeParams;

constexpr int kVersion = 100;     // 0.1.0
constexpr int kConsumerWarps = 4;       // each takes 16 positions of a pipeline stage
constexpr int kTile = 16 * kConsumerWarps;
inline int tile_rows() { return kTile; }

constexpr int kClusterCtas = 8;         // cluster size of the fused merge
constexpr int kMaxUnits = 1 << 16;      // fused-merge counters kept per device
constexpr size_t kCounterBytes = size_t(kMaxUnits) * sizeof(int);

thread_local int t_last_cuda = 0;
std::atomic<unsigned long long> g_launches{0};   // kernels launched (or captured) by this library
std::atomic<int> g_overlap{0};                   // fr_set_launch_overlap

int cuda_fail(cudaError_t e) {
    t_last_cuda = static_cast<int>(e);
    return FR_ERR_CUDA;
}

struct DeviceState {
    int sm_count = 0;
    int* err = nullptr;          // device error word
    void* ws = nullptr;          // split partial states
    size_t ws_bytes = 0;
    uint32_t attr_done = 0;      // bit per kernel instantiation: smem attribute set
    int occupancy[8] = {0};      // CTAs/SM per instantiation (0 = not queried)
    int persist_occ[4] = {0};    // CTAs/SM of the persistent batched kernels
    int resident[4][5] = {{-1, -1, -1, -1, -1}, {-1, -1, -1, -1, -1}, {-1, -1, -1, -1, -1},
                          {-1, -1, -1, -1, -1}};   // co-resident clusters per (slot, log2 size)
    int resident_g[4][2] = {{-1, -1}, {-1, -1}, {-1, -1}, {-1, -1}};   // grouped form, 8 / 16
};

std::mutex g_mu;
std::unordered_map<int, DeviceState> g_dev;

// Returns the current device's state, creating it (cudaMalloc of the error
// word) on first use.  First use must therefore happen outside graph capture.
int get_state(DeviceState** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& st = g_dev[dev];
    if (!st.err) {
        e = cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e);
        e = cudaMalloc(&st.err, sizeof(int));
        if (e != cudaSuccess) { st.err = nullptr; return cuda_fail(e); }
        e = cudaMemset(st.err, 0, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e);
    }
    *out = &st;
    return FR_OK;
}

bool is_capturing(cudaStream_t s) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) return false;
    return cs != cudaStreamCaptureStatusNone;
}

int ensure_workspace(DeviceState* st, size_t bytes, cudaStream_t s) {
    if (bytes <= st->ws_bytes) return FR_OK;
    if (is_capturing(s)) return FR_ERR_WORKSPACE;
    std::lock_guard<std::mutex> lk(g_mu);
    if (bytes <= st->ws_bytes) return FR_OK;
    if (st->ws) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e);
        cudaFree(st->ws);
        st->ws = nullptr;
        st->ws_bytes = 0;
    }
    const size_t grow = bytes + bytes / 4;
    cudaError_t e = cudaMalloc(&st->ws, grow);
    if (e != cudaSuccess) { st->ws = nullptr; return cuda_fail(e); }
    // The fused merge's counters (start of the buffer) must be zero between calls.
    e = cudaMemset(st->ws, 0, std::min(grow, kCounterBytes));
    if (e != cudaSuccess) return cuda_fail(e);
    st->ws_bytes = grow;
    return FR_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int env_int(const char* name, int dflt);

// ------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// View of a cache [rows][Hkv][D] fp16 as a 4-D tensor [rows][Hkv][D/64][64]
// (innermost first below), box = 64 dims x box_rows (default tile_rows())
// rows of one kv head, 128-byte swizzle.  Rows >= `rows` read as zeros.
int encode_kv_map(CUtensorMap* map, const void* base, int head_dim, int num_kv_heads,
                  long long rows, int box_rows = 0) {
    const int kTile = box_rows > 0 ? box_rows : tile_rows();
    std::memset(map, 0, sizeof(*map));
    if (rows <= 0) return FR_OK;                      // never read (empty range)
    if (rows > (1LL << 31)) return FR_ERR_INVALID_ARG;
    auto fn = encode_fn();
    if (!fn) return cuda_fail(cudaErrorNotSupported);
    const cuuint64_t dims[4] = {64, (cuuint64_t)(head_dim / 64), (cuuint64_t)num_kv_heads,
                                (cuuint64_t)rows};
    const cuuint64_t strides[3] = {128, (cuuint64_t)head_dim * 2,
                                   (cuuint64_t)num_kv_heads * head_dim * 2};
    const cuuint32_t box[4] = {64, 1, 1, (cuuint32_t)kTile};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    static const int promo = env_int("FORGERT_L2_PROMO", 3);
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    static_cast<CUtensorMapL2promotion>(promo & 3),
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cuda_fail(cudaErrorInvalidValue);
    return FR_OK;
}

// ------------------------------------------------------------- kernel table
// One instantiation per (head_dim, head tile, cluster size).  Stages of
// 16 KB (D=64) / 32 KB (D=128) K+V; the ring keeps 96 KB in flight per CTA,
// so two CTAs fit on an SM.
template <int D> struct Stages;
template <> struct Stages<64> { static constexpr int value = 6; };
template <> struct Stages<128> { static constexpr int value = 3; };

template <int D, int NT>
constexpr int kernel_slot() { return (D == 64 ? 0 : 2) + (NT - 1); }

template <int D, int NT, int CL, bool PAGED = false>
auto kernel_ptr() {
    return fr::split_decode_kernel<D, NT, kTile, Stages<D>::value, kConsumerWarps, CL, PAGED>;
}

template <int D, int NT>
using SmemOf = fr::SplitSmem<D, NT, kTile, Stages<D>::value, kConsumerWarps>;

// Grouped form of the fused single-sequence kernel: two groups of four
// consumer warps take alternate tiles (each group owns half the ring's
// stages: 4 at D=128, one CTA per SM), so a CTA consumes its prefetched
// tiles at twice the rate.  Used for small grids (at most one CTA per two
// SMs, the next call's CTAs fitting on the other SMs) of at least two tiles
// per CTA, with clusters of 8 or 16.
template <int D> struct StagesG;
template <> struct StagesG<64> { static constexpr int value = 6; };
template <> struct StagesG<128> { static constexpr int value = 4; };
constexpr int kGroupedWarps = 2 * kConsumerWarps;

template <int D, int NT, int CL>
auto kernel_ptr_g() {
    return fr::split_decode_kernel<D, NT, kTile, StagesG<D>::value, kGroupedWarps, CL, false>;
}

template <int D, int NT>
using SmemOfG = fr::SplitSmem<D, NT, kTile, StagesG<D>::value, kGroupedWarps>;

template <int D, int NT, int CL>
int set_smem_attr() {
    auto set = [](auto fn, size_t bytes) -> int {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(bytes));
        if (e == cudaSuccess && CL > 8)        // 16-CTA clusters are a non-portable size
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e == cudaSuccess ? FR_OK : cuda_fail(e);
    };
    int rc = set(kernel_ptr<D, NT, CL, false>(), SmemOf<D, NT>::kBytes);
    if (rc == FR_OK) rc = set(kernel_ptr<D, NT, CL, true>(), SmemOf<D, NT>::kBytes);
    if constexpr (CL >= 8) {
        if (rc == FR_OK) rc = set(kernel_ptr_g<D, NT, CL>(), SmemOfG<D, NT>::kBytes);
    }
    return rc;
}

// Guards the per-device attribute bits, occupancy and co-residency caches:
// two host threads making their first call on one device must not race on
// them.
std::mutex g_prep_mu;

template <int D, int NT>
int prepare_kernel(DeviceState* st) {
    constexpr int slot = kernel_slot<D, NT>();
    std::lock_guard<std::mutex> lk(g_prep_mu);
    if (!(st->attr_done & (1u << slot))) {
        int rc = set_smem_attr<D, NT, 1>();
        if (rc == FR_OK) rc = set_smem_attr<D, NT, 2>();
        if (rc == FR_OK) rc = set_smem_attr<D, NT, 4>();
        if (rc == FR_OK) rc = set_smem_attr<D, NT, 8>();
        if (rc == FR_OK) rc = set_smem_attr<D, NT, 16>();
        if (rc != FR_OK) return rc;
        int n = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &n, kernel_ptr<D, NT, 1>(), 32 * (kConsumerWarps + 1), SmemOf<D, NT>::kBytes);
        st->occupancy[slot] = (e == cudaSuccess && n > 0) ? n : 1;
        st->attr_done |= (1u << slot);
    }
    return FR_OK;
}

// Launch with optional cluster shape and programmatic dependent launch.
template <int D, int NT, int CL, bool PAGED>
int launch_split(const DecodeParams& p, dim3 grid, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * (kConsumerWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = SmemOf<D, NT>::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attrs[2];
    unsigned n = 0;
    if (CL > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = 1;
        attrs[n].val.clusterDim.y = CL;
        attrs[n].val.clusterDim.z = 1;
        ++n;
    }
    if (pdl) {
        attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel_ptr<D, NT, CL, PAGED>(), p);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return FR_OK;
}

// Co-resident clusters of 8 or 16 CTAs of the grouped form (cached).
int resident_clusters_g(int D, int nt, int cl, DeviceState* st) {
    const int slot = (D == 64 ? 0 : 2) + (nt - 1);
    std::lock_guard<std::mutex> lk(g_prep_mu);
    int& cached = st->resident_g[slot][cl == 16 ? 1 : 0];
    if (cached >= 0) return cached;
    const void* fn = nullptr;
    size_t smem = 0;
    if (D == 64) {
        fn = nt == 1 ? (cl == 16 ? (const void*)kernel_ptr_g<64, 1, 16>() : (const void*)kernel_ptr_g<64, 1, 8>())
                     : (cl == 16 ? (const void*)kernel_ptr_g<64, 2, 16>() : (const void*)kernel_ptr_g<64, 2, 8>());
        smem = nt == 1 ? SmemOfG<64, 1>::kBytes : SmemOfG<64, 2>::kBytes;
    } else {
        fn = nt == 1 ? (cl == 16 ? (const void*)kernel_ptr_g<128, 1, 16>() : (const void*)kernel_ptr_g<128, 1, 8>())
                     : (cl == 16 ? (const void*)kernel_ptr_g<128, 2, 16>() : (const void*)kernel_ptr_g<128, 2, 8>());
        smem = nt == 1 ? SmemOfG<128, 1>::kBytes : SmemOfG<128, 2>::kBytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, cl, 1);
    cfg.blockDim = dim3(32 * (kGroupedWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = cl;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n < 0) {
        cudaGetLastError();
        n = 0;
    }
    cached = n;
    return n;
}

// The grouped form (clusters of 8 or 16, contiguous caches).
template <int D, int NT, int CL>
int launch_split_g(const DecodeParams& p, dim3 grid, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * (kGroupedWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = SmemOfG<D, NT>::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attrs[2];
    unsigned n = 0;
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = CL;
    attrs[n].val.clusterDim.z = 1;
    ++n;
    if (pdl) {
        attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel_ptr_g<D, NT, CL>(), p);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return FR_OK;
}

template <int D>
int launch_grouped(const DecodeParams& p, int nt, int cl, dim3 grid, cudaStream_t s, bool pdl) {
    if (nt == 1)
        return cl == 16 ? launch_split_g<D, 1, 16>(p, grid, s, pdl) : launch_split_g<D, 1, 8>(p, grid, s, pdl);
    return cl == 16 ? launch_split_g<D, 2, 16>(p, grid, s, pdl) : launch_split_g<D, 2, 8>(p, grid, s, pdl);
}

template <int D, int NT, bool PAGED>
int launch_split_nt(const DecodeParams& p, int cl, dim3 grid, cudaStream_t s, bool pdl) {
    switch (cl) {
        case 16: return launch_split<D, NT, 16, PAGED>(p, grid, s, pdl);
        case 8: return launch_split<D, NT, 8, PAGED>(p, grid, s, pdl);
        case 4: return launch_split<D, NT, 4, PAGED>(p, grid, s, pdl);
        case 2: return launch_split<D, NT, 2, PAGED>(p, grid, s, pdl);
        default: return launch_split<D, NT, 1, PAGED>(p, grid, s, pdl);
    }
}

// The paged instantiation is chosen by p.block_table.
template <int D>
int launch_split_any(const DecodeParams& p, int nt, int cl, dim3 grid, cudaStream_t s, bool pdl) {
    if (p.block_table)
        return nt == 1 ? launch_split_nt<D, 1, true>(p, cl, grid, s, pdl)
                       : launch_split_nt<D, 2, true>(p, cl, grid, s, pdl);
    return nt == 1 ? launch_split_nt<D, 1, false>(p, cl, grid, s, pdl)
                   : launch_split_nt<D, 2, false>(p, cl, grid, s, pdl);
}

struct Plan {
    int nt = 1;            // 8-head tiles per CTA (1 or 2)
    int head_groups = 1;   // CTAs per kv head along the query group
    int num_splits = 1;
    int split_len = 0;     // positions per split, multiple of tile_rows()
};

// Splits the longest sequence so the grid fills the GPU about `waves` times:
// units = batch * kv_heads * head_groups CTAs per split.
Plan make_plan(int sm_count, int occ, int batch, int num_kv_heads, int group, int max_kv_len,
               int waves) {
    const int kTile = tile_rows();
    Plan pl;
    pl.nt = group <= 8 ? 1 : 2;
    pl.head_groups = (group + 8 * pl.nt - 1) / (8 * pl.nt);
    const long long units = (long long)batch * num_kv_heads * pl.head_groups;
    const int tiles = std::max(1, (max_kv_len + kTile - 1) / kTile);
    const long long slots = (long long)sm_count * occ * waves;
    long long want = std::max<long long>(1, slots / std::max<long long>(1, units));
    want = std::min<long long>(want, tiles);
    const int tps = (int)((tiles + want - 1) / want);
    pl.split_len = tps * kTile;
    pl.num_splits = (tiles + tps - 1) / tps;
    return pl;
}

template <int D>
int launch_merge(const float* ml, const float* acc, int num_states, fr::MergeStrides st, int rows,
                 __half* out, float* out_ml, float* out_acc, int mode, cudaStream_t s,
                 bool pdl = false) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, 1, 1);
    cfg.blockDim = dim3(32 * fr::kMergeWarps, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fr::lse_merge_kernel<D>, ml, acc, num_states, st, out,
                                       out_ml, out_acc, mode);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return FR_OK;
}

size_t partial_bytes(long long rows, int splits, int head_dim) {
    return (size_t)rows * splits * (2 + head_dim) * sizeof(float);
}

int check_heads(int num_heads, int num_kv_heads, int head_dim) {
    if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return FR_ERR_INVALID_ARG;
    if (head_dim != 64 && head_dim != 128) return FR_ERR_UNSUPPORTED;
    return FR_OK;
}

// Tuning knobs (read once): FORGERT_SLOTS_PER_SM caps the CTAs per SM the
// planner fills (default: the occupancy limit); FORGERT_CLUSTER_MIN_SPLITS is
// the split count from which the fused merge uses clusters (default 8, 0 =
// never).
int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

// Single-sequence calls (waves == 1) plan one CTA per SM: with the other
// slot free, the next call's CTAs can become resident and start streaming
// K/V while this call merges (programmatic dependent launch).
int slots_per_sm(int occ, int waves) {
    static const int cap = env_int("FORGERT_SLOTS_PER_SM", 0);
    if (cap > 0) return std::min(cap, occ);
    return waves == 1 ? 1 : occ;
}


int max_splits() {
    static const int v = env_int("FORGERT_MAX_SPLITS", 0);
    return v;
}

// FORGERT_ONE_CLUSTER_TILES: the most tiles per CTA for which a unit is
// covered by one 16-CTA cluster (default 4; 0 = never).
// FORGERT_MAX_CLUSTER: largest cluster of the multi-cluster plans (8 or 16).
int max_cluster() {
    static const int v = env_int("FORGERT_MAX_CLUSTER", 8);
    return v;
}

// CTA waves a batched or paged call plans for (ragged batches: several waves
// of shorter splits balance the tail).
int batch_waves() {
    static const int v = std::min(16, std::max(2, env_int("FORGERT_BATCH_WAVES", 4)));
    return v;
}

int one_cluster_tiles() {
    static const int v = env_int("FORGERT_ONE_CLUSTER_TILES", 4);
    return v;
}

int cluster_min_splits() {
    static const int v = env_int("FORGERT_CLUSTER_MIN_SPLITS", kClusterCtas);
    return v;
}

int plan_for(DeviceState* st, int head_dim, int batch, int num_kv_heads, int group,
             int max_kv_len, int waves, Plan* pl) {
    const int nt = group <= 8 ? 1 : 2;
    const int kTile = tile_rows();
    int rc;
    rc = head_dim == 64 ? (nt == 1 ? prepare_kernel<64, 1>(st) : prepare_kernel<64, 2>(st))
                        : (nt == 1 ? prepare_kernel<128, 1>(st) : prepare_kernel<128, 2>(st));
    if (rc != FR_OK) return rc;
    const int slot = (head_dim == 64 ? 0 : 2) + (nt - 1);
    const int occ = slots_per_sm(st->occupancy[slot], waves);
    *pl = make_plan(st->sm_count, occ, batch, num_kv_heads, group, max_kv_len, waves);
    const int cap = max_splits();
    if (cap > 0 && pl->num_splits > cap) {
        const int tiles = std::max(1, (max_kv_len + kTile - 1) / kTile);
        const int tps = (tiles + cap - 1) / cap;
        pl->split_len = tps * kTile;
        pl->num_splits = (tiles + tps - 1) / tps;
    }
    return FR_OK;
}

// Clusters of `cl` CTAs (or CTAs, cl == 1) of the split kernel that can be
// resident on the device at once.
int query_resident_clusters(int D, int nt, int cl, DeviceState* st);

int resident_clusters(int D, int nt, int cl, DeviceState* st) {
    const int slot = (D == 64 ? 0 : 2) + (nt - 1);
    const int li = cl >= 16 ? 4 : cl >= 8 ? 3 : cl >= 4 ? 2 : cl >= 2 ? 1 : 0;
    std::lock_guard<std::mutex> lk(g_prep_mu);
    int& cached = st->resident[slot][li];
    if (cached < 0) cached = query_resident_clusters(D, nt, cl, st);
    return cached;
}

int query_resident_clusters(int D, int nt, int cl, DeviceState* st) {
    const int slot = (D == 64 ? 0 : 2) + (nt - 1);
    if (cl == 1) return st->sm_count * std::max(1, st->occupancy[slot]);
    const void* fn = nullptr;
    size_t smem = 0;
    auto pick = [&](auto kfn, size_t bytes) { fn = reinterpret_cast<const void*>(kfn); smem = bytes; };
    auto choose = [&](auto k16, auto k8, auto k4, auto k2, size_t bytes) {
        pick(cl == 16 ? k16 : cl == 8 ? k8 : cl == 4 ? k4 : k2, bytes);
    };
    if (D == 64) {
        if (nt == 1) choose(kernel_ptr<64, 1, 16>(), kernel_ptr<64, 1, 8>(), kernel_ptr<64, 1, 4>(), kernel_ptr<64, 1, 2>(), SmemOf<64, 1>::kBytes);
        else choose(kernel_ptr<64, 2, 16>(), kernel_ptr<64, 2, 8>(), kernel_ptr<64, 2, 4>(), kernel_ptr<64, 2, 2>(), SmemOf<64, 2>::kBytes);
    } else {
        if (nt == 1) choose(kernel_ptr<128, 1, 16>(), kernel_ptr<128, 1, 8>(), kernel_ptr<128, 1, 4>(), kernel_ptr<128, 1, 2>(), SmemOf<128, 1>::kBytes);
        else choose(kernel_ptr<128, 2, 16>(), kernel_ptr<128, 2, 8>(), kernel_ptr<128, 2, 4>(), kernel_ptr<128, 2, 2>(), SmemOf<128, 2>::kBytes);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, cl, 1);
    cfg.blockDim = dim3(32 * (kConsumerWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = cl;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// ------------------------------------------------ persistent batched path
// fr_decode_attn_batched runs the persistent stream-K kernel
// (batched_kernels.cuh) when the batch fits its shared-memory length prefix;
// FORGERT_BATCHED_KERNEL=split selects the split kernel's grid instead
// (read once).  FORGERT_PERSIST_CTAS_PER_SM caps the CTAs per SM of the
// persistent grid (default: as many as fit); FORGERT_PERSIST_MIN_TILES
// (default 8, 0 = off) is the fewest tiles per CTA the kernel aims for
// before it leaves CTAs idle (never fewer than one CTA per SM).
template <int D, int NT>
using PersistOf = fr::PersistSmem<D, NT, kTile, Stages<D>::value, kConsumerWarps>;

template <int D, int NT>
auto persist_ptr() {
    return fr::persistent_decode_kernel<D, NT, kTile, Stages<D>::value, kConsumerWarps>;
}

bool persistent_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("FORGERT_BATCHED_KERNEL");
        return !(v && std::strcmp(v, "split") == 0);
    }();
    return on;
}

int persist_ctas_per_sm(int occ) {
    static const int cap = env_int("FORGERT_PERSIST_CTAS_PER_SM", 0);
    return cap > 0 ? std::min(cap, occ) : occ;
}

// Attribute bits 12..15 of attr_done; occupancy in persist_occ[slot].
template <int D, int NT>
int prepare_persistent(DeviceState* st, int* occ) {
    constexpr int slot = kernel_slot<D, NT>();
    std::lock_guard<std::mutex> lk(g_prep_mu);
    const uint32_t bit = 1u << (12 + slot);
    if (!(st->attr_done & bit)) {
        cudaError_t e = cudaFuncSetAttribute(persist_ptr<D, NT>(),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(PersistOf<D, NT>::kBytes));
        if (e != cudaSuccess) return cuda_fail(e);
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, persist_ptr<D, NT>(),
                                                          32 * (kConsumerWarps + 1),
                                                          PersistOf<D, NT>::kBytes);
        st->persist_occ[slot] = (e == cudaSuccess && n > 0) ? n : 1;
        st->attr_done |= bit;
    }
    *occ = st->persist_occ[slot];
    return FR_OK;
}

template <int D, int NT>
int launch_persistent(const DecodeParams& p, int ctas, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, 1, 1);
    cfg.blockDim = dim3(32 * (kConsumerWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = PersistOf<D, NT>::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, persist_ptr<D, NT>(), p);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

// Grid and workspace of a persistent call: C co-resident CTAs (no more than
// the tiles the call can have), 2 partial slots of GP x (D + 2) floats each.
struct PersistPlan {
    int nt = 1, head_groups = 1, ctas = 0;
    size_t ws_bytes = 0;
};

int persistent_plan(DeviceState* st, int D, int batch, int num_kv_heads, int group,
                    int max_kv_len, PersistPlan* pp) {
    PersistPlan pl;
    pl.nt = group <= 8 ? 1 : 2;
    pl.head_groups = (group + 8 * pl.nt - 1) / (8 * pl.nt);
    int occ = 1;
    const int rc = D == 64 ? (pl.nt == 1 ? prepare_persistent<64, 1>(st, &occ)
                                         : prepare_persistent<64, 2>(st, &occ))
                           : (pl.nt == 1 ? prepare_persistent<128, 1>(st, &occ)
                                         : prepare_persistent<128, 2>(st, &occ));
    if (rc != FR_OK) return rc;
    const long long upb = (long long)num_kv_heads * pl.head_groups;
    const long long max_tiles =
        (long long)batch * upb * std::max(1, (max_kv_len + kTile - 1) / kTile);
    const long long slots = (long long)st->sm_count * persist_ctas_per_sm(occ);
    pl.ctas = (int)std::max<long long>(1, std::min(slots, max_tiles));
    const int gp = 8 * pl.nt;
    pl.ws_bytes = kCounterBytes + (size_t)2 * pl.ctas * gp * (D + 2) * sizeof(float);
    *pp = pl;
    return FR_OK;
}

bool persistent_fits(int batch, int num_kv_heads, int group, int max_kv_len) {
    if (!persistent_enabled() || batch > fr::kPersistMaxBatch) return false;
    const int nt = group <= 8 ? 1 : 2;
    const long long upb = (long long)num_kv_heads * ((group + 8 * nt - 1) / (8 * nt));
    const long long units = (long long)batch * upb;
    const long long tiles = units * std::max(1, (max_kv_len + kTile - 1) / kTile);
    return units <= kMaxUnits && tiles < (1LL << 30);
}

int run_persistent(DecodeParams p, int head_dim, int batch, int max_kv_len, __half* out,
                   cudaStream_t s) {
    DeviceState* st = nullptr;
    int rc = get_state(&st);
    if (rc != FR_OK) return rc;
    const int group = p.H / p.Hkv;
    PersistPlan pl;
    rc = persistent_plan(st, head_dim, batch, p.Hkv, group, max_kv_len, &pl);
    if (rc != FR_OK) return rc;
    rc = ensure_workspace(st, pl.ws_bytes, s);
    if (rc != FR_OK) return rc;
    p.G = group;
    p.head_groups = pl.head_groups;
    p.batch = batch;
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
    p.err = st->err;
    p.out = out;
    p.counters = static_cast<int*>(st->ws);
    p.part_ml = reinterpret_cast<float*>(static_cast<char*>(st->ws) + kCounterBytes);
    p.part_acc = p.part_ml + (size_t)2 * pl.ctas * 8 * pl.nt * 2;
    static const int evict_normal = env_int("FORGERT_EVICT_NORMAL", 0);
    p.evict_normal = evict_normal;
    const bool pdl = s != nullptr;
    p.prefetch_meta = (pdl && g_overlap.load(std::memory_order_relaxed)) ? 1 : 0;
    static const int min_tiles = env_int("FORGERT_PERSIST_MIN_TILES", 8);
    p.min_tiles_per_cta = std::max(0, min_tiles);
    p.min_ctas = st->sm_count;
    // Partition cost of starting an item and of merging a unit, in tile
    // times (FORGERT_PERSIST_ITEM_COST / _MERGE_COST, read once).
    static const int item_cost = std::max(0, env_int("FORGERT_PERSIST_ITEM_COST", 4));
    static const int merge_cost = std::max(0, env_int("FORGERT_PERSIST_MERGE_COST", 4));
    p.item_cost = item_cost;
    p.merge_cost = merge_cost;
    static const int trace_plan = env_int("FORGERT_TRACE_PLAN", 0);
    if (trace_plan)
        std::fprintf(stderr, "[forgert] persistent D=%d batch=%d units=%d ctas=%d prefetch=%d\n",
                     head_dim, batch, batch * p.Hkv * pl.head_groups, pl.ctas, p.prefetch_meta);
    if (head_dim == 64)
        return pl.nt == 1 ? launch_persistent<64, 1>(p, pl.ctas, s, pdl)
                          : launch_persistent<64, 2>(p, pl.ctas, s, pdl);
    return pl.nt == 1 ? launch_persistent<128, 1>(p, pl.ctas, s, pdl)
                      : launch_persistent<128, 2>(p, pl.ctas, s, pdl);
}

// Shared driver of the decode-family entry points.  `p` carries the tensor
// maps and the sequence geometry.
//   final_out != nullptr : write fp16 output
//   state_ml  != nullptr : write one merged (m, l, acc) state per head row
// Splits are merged inside the split kernel (clusters of kClusterCtas CTAs
// through DSMEM, then the last cluster per kv head); a second launch is
// needed only when there are more (b, kv head, head group) units than
// counters.
int run_decode(DecodeParams p, int head_dim, int batch, int max_kv_len, __half* final_out,
               float* state_ml, float* state_acc, int waves, cudaStream_t s) {
    DeviceState* st = nullptr;
    int rc = get_state(&st);
    if (rc != FR_OK) return rc;
    const int D = head_dim;
    const int group = p.H / p.Hkv;
    Plan pl;
    rc = plan_for(st, D, batch, p.Hkv, group, max_kv_len, waves, &pl);
    if (rc != FR_OK) return rc;
    const long long units = (long long)batch * p.Hkv * pl.head_groups;
    // Cluster size: the largest of 8/4/2 whose whole clusters cover nearly as
    // many splits as the plan wants (every SM busy matters more than the
    // merge depth); fewer than cluster_min_splits() splits merge without
    // clusters (batched calls hide that merge behind other units).
    const int cmin = cluster_min_splits();
    int cl = 1;
    // Short ranges of a few units: one cluster of 16 per unit with at most
    // one_cluster_tiles() tiles per CTA needs no merge across clusters, which
    // costs more than the extra tiles (single-sequence calls only).
    const int kTileRows = tile_rows();
    const int tiles_u = std::max(1, (max_kv_len + kTileRows - 1) / kTileRows);
    const int oct = one_cluster_tiles();
    const bool one_cluster16 = waves == 1 && oct > 0 && tiles_u > 8 && tiles_u <= 16 * oct &&
                               units * 16 <= st->sm_count &&
                               resident_clusters(D, pl.nt, 16, st) >= units;
    if (one_cluster16) {
        cl = 16;
        const int tps = (tiles_u + 15) / 16;
        pl.split_len = tps * kTileRows;
        pl.num_splits = (tiles_u + tps - 1) / tps;
    } else if (cmin > 0 && pl.num_splits >= cmin) {
        const int want = pl.num_splits;
        cl = (max_cluster() >= 16 && want >= 16 && resident_clusters(D, pl.nt, 16, st) > 0) ? 16 : 8;
        for (int c : {8, 4, 2})
            if (c < cl && (want / c) * c * 20 >= (want / cl) * cl * 21) cl = c;   // > 5% more splits
        const int kTile = tile_rows();
        const int tiles = std::max(1, (max_kv_len + kTile - 1) / kTile);
        const int nsp = std::max(cl, want / cl * cl);
        const int tps = (tiles + nsp - 1) / nsp;
        pl.split_len = tps * kTile;
        pl.num_splits = (tiles + tps - 1) / tps;
    }
    const bool fused = units * cl <= kMaxUnits;      // one counter per (unit, cluster rank)
    if (p.xworld > 0) {
        // The exchange waits inside the kernel for the other GPUs, which wait
        // for this one: every cluster of the grid must be resident at once.
        if (!fused) return FR_ERR_UNSUPPORTED;
        const int resident = resident_clusters(D, pl.nt, cl, st);
        const long long max_splits_res = (long long)(resident / std::max<long long>(1, units)) * cl;
        if (max_splits_res < cl) return FR_ERR_UNSUPPORTED;
        if (pl.num_splits > max_splits_res) {
            const int kTile = tile_rows();
            const int tiles = std::max(1, (max_kv_len + kTile - 1) / kTile);
            const int tps = (int)((tiles + max_splits_res - 1) / max_splits_res);
            pl.split_len = tps * kTile;
            pl.num_splits = (tiles + tps - 1) / tps;
        }
    }
    const int splits = (pl.num_splits + cl - 1) / cl * cl;     // pads at most one cluster
    p.G = group;
    p.split_len = pl.split_len;
    p.num_splits = splits;
    p.head_groups = pl.head_groups;
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
    p.err = st->err;
    static const int evict_normal = env_int("FORGERT_EVICT_NORMAL", 0);
    p.evict_normal = evict_normal;
    const bool pdl = s != nullptr;
    const long long rows = (long long)batch * p.H;
    if (final_out && splits == 1 && p.xworld == 0) {
        p.write_final = 1;
        p.out = final_out;
    } else {
        const int slots = fused ? splits / cl : splits;
        rc = ensure_workspace(st, kCounterBytes + partial_bytes(rows, slots, D), s);
        if (rc != FR_OK) return rc;
        p.part_slots = slots;
        p.part_ml = reinterpret_cast<float*>(static_cast<char*>(st->ws) + kCounterBytes);
        p.part_acc = p.part_ml + rows * slots * 2;
        if (fused) {
            p.counters = static_cast<int*>(st->ws);
            p.out = final_out;
            p.out_ml = state_ml;
            p.out_acc = state_acc;
        }
    }
    dim3 grid(p.Hkv * pl.head_groups, splits, batch);
    // Grouped consumers (two tiles at a time per CTA): a fused single-sequence
    // call on contiguous caches, clusters of 8 or 16, at least two tiles per
    // CTA, and a grid of at most one CTA per two SMs (FORGERT_GROUPED, read
    // once: 0 = never, 2 = whatever the grid size).
    static const int grouped_on = env_int("FORGERT_GROUPED", 1);
    const long long ctas = (long long)grid.x * grid.y * grid.z;
    const bool grouped = grouped_on && waves == 1 && p.counters && !p.block_table &&
                         p.xworld == 0 && (cl == 8 || cl == 16) &&
                         pl.split_len >= 2 * kTile && (grouped_on == 2 || 2 * ctas <= st->sm_count) &&
                         (long long)resident_clusters_g(D, pl.nt, cl, st) * cl >= ctas;
    static const int trace_plan = env_int("FORGERT_TRACE_PLAN", 0);
    if (trace_plan)
        std::fprintf(stderr, "[forgert] plan D=%d batch=%d units=%lld splits=%d split_len=%d "
                     "cluster=%d fused=%d xworld=%d grouped=%d grid=(%u,%u,%u)\n", D, batch,
                     units, splits, pl.split_len, cl, (int)fused, p.xworld, (int)grouped, grid.x,
                     grid.y, grid.z);
    if (grouped)
        return D == 64 ? launch_grouped<64>(p, pl.nt, cl, grid, s, pdl)
                       : launch_grouped<128>(p, pl.nt, cl, grid, s, pdl);
    rc = D == 64 ? launch_split_any<64>(p, pl.nt, cl, grid, s, pdl)
                 : launch_split_any<128>(p, pl.nt, cl, grid, s, pdl);
    if (rc != FR_OK || p.write_final || p.counters) return rc;
    // unfused: a separate merge launch
    const int mode = final_out ? 0 : 1;
    const fr::MergeStrides ms{2LL * splits, 2, (long long)splits * D, D};
    return D == 64 ? launch_merge<64>(p.part_ml, p.part_acc, splits, ms, (int)rows, final_out,
                                      state_ml, state_acc, mode, s, pdl)
                   : launch_merge<128>(p.part_ml, p.part_acc, splits, ms, (int)rows, final_out,
                                       state_ml, state_acc, mode, s, pdl);
}

// Causal prefill: grid (heads, query tiles of 64), programmatic dependent
// launch on non-default streams.  The shared-memory attribute is set once per
// device (bits 8/9 of attr_done).
template <int D>
int launch_prefill(DeviceState* st, const fr::PrefillParams& pp, cudaStream_t s) {
    constexpr int kStages = Stages<D>::value;
    using PS = fr::PrefillSmem<D, kStages>;
    auto fn = fr::prefill_kernel<D, kStages>;
    const uint32_t bit = 1u << (D == 64 ? 8 : 9);
    std::unique_lock<std::mutex> lk(g_prep_mu);
    if (!(st->attr_done & bit)) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(PS::kBytes));
        if (e != cudaSuccess) return cuda_fail(e);
        st->attr_done |= bit;
    }
    lk.unlock();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pp.H, (pp.T + PS::kTile - 1) / PS::kTile, 1);
    cfg.blockDim = dim3(160, 1, 1);
    cfg.dynamicSmemBytes = PS::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = s != nullptr ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, pp);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

// Split plan of the tcgen05 prefill: K/V tiles per work unit (0 = one unit
// per query tile), units and partial slots per head.  Causal query tiles
// differ in length (the last has the most K/V tiles); when the longest one
// outlasts the average load of a CTA slot (two per SM), the K/V ranges are
// cut into units of half or a quarter of the longest range, merged by the
// last unit of a query tile to finish.  The choice minimises the estimated
// makespan max(longest unit, total work / slots), counting a fixed cost of
// four tile times per unit and a merge of one tile time per unit of the
// query tile for split units (fitted to B200 measurements of T 512..8192,
// H 4..28); each finer split must gain 15 % on the estimate.
// FORGERT_PREFILL_CHUNK forces the size (0 = never split), read per call.
struct PrefillPlan {
    int chunk_tiles = 0;
    int units_per_head = 0;
    int slots_per_head = 0;
};

PrefillPlan prefill_plan(int T, int H, int sm_count) {
    constexpr int kRows = 128, kTile = 64;
    constexpr double kFixed = 4.0, kMerge = 2.0;     // in K/V tile times
    const int nq = (T + kRows - 1) / kRows;
    auto tiles = [&](int qt) { return (std::min(qt * kRows + kRows, T) + kTile - 1) / kTile; };
    const int nmax = tiles(nq - 1);
    const double slots = 2.0 * sm_count;
    // estimated makespan of chunk size ct (ct >= nmax: unsplit)
    auto estimate = [&](int ct) {
        double longest = 0, total = 0;
        for (int qt = 0; qt < nq; ++qt) {
            const int n = tiles(qt);
            if (ct >= n) {
                longest = std::max(longest, n + kFixed);
                total += n + kFixed;
            } else {
                const int nc = (n + ct - 1) / ct;
                for (int j = 0; j < n; j += ct) {
                    const double w = std::min(ct, n - j) + kFixed + kMerge * nc / 2;
                    longest = std::max(longest, w);
                    total += w;
                }
            }
        }
        return std::max(longest, total * H / slots);
    };
    PrefillPlan pl;
    pl.units_per_head = nq;
    const int lo = std::max(1, (nmax + fr::kMaxPrefillChunks - 1) / fr::kMaxPrefillChunks);
    int ct = 0;
    const int forced = env_int("FORGERT_PREFILL_CHUNK", -1);
    if (forced >= 0) {
        ct = forced > 0 ? std::max(forced, lo) : 0;
    } else if ((long long)H * nq <= kMaxUnits) {
        const double base = estimate(nmax);
        // When the total work per slot bounds the estimate, splitting only
        // adds merges: search only when the longest query tile bounds it.
        if (base <= nmax + kFixed) {
            double best = base;
            for (int parts = 2; parts <= fr::kMaxPrefillChunks; parts *= 2) {
                const int c = (nmax + parts - 1) / parts;
                if (c >= nmax) continue;
                const double e = estimate(c);
                if (e < 0.85 * best) {       // each finer split must gain 15 %
                    best = e;
                    ct = c;
                }
            }
        }
    }
    if (ct <= 0 || ct >= nmax || (long long)H * nq > kMaxUnits) return pl;
    pl.chunk_tiles = ct;
    pl.units_per_head = 0;
    for (int qt = 0; qt < nq; ++qt) {
        const int nc = (tiles(qt) + ct - 1) / ct;
        pl.units_per_head += nc;
        if (nc > 1) pl.slots_per_head += nc;
    }
    return pl;
}

size_t prefill_partial_bytes(const PrefillPlan& pl, int H, int D) {
    return (size_t)H * pl.slots_per_head * 128 * (D + 2) * sizeof(float);
}

// Causal prefill on tcgen05: grid (heads, work units), 192 threads, two CTAs
// per SM, each with 256 TMEM columns and at most half of the shared memory
// (attribute bits 10/11 of attr_done).  A split plan needs workspace for the
// partial states; inside a graph capture that cannot grow it, the call runs
// unsplit instead.
template <int D>
int launch_prefill_tc(DeviceState* st, fr::PrefillParams pp, cudaStream_t s) {
    constexpr int kStages = D == 64 ? 4 : 2;
    using PS = fr::PrefillTcSmem<D, kStages>;
    static_assert(2 * PS::kBytes <= 228 * 1024 && 3 * PS::kBytes > 228 * 1024,
                  "exactly two CTAs per SM: their TMEM columns fill the SM");
    auto fn = fr::prefill_tc_kernel<D, kStages>;
    const uint32_t bit = 1u << (D == 64 ? 10 : 11);
    std::unique_lock<std::mutex> lk(g_prep_mu);
    if (!(st->attr_done & bit)) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(PS::kBytes));
        if (e != cudaSuccess) return cuda_fail(e);
        st->attr_done |= bit;
    }
    lk.unlock();
    const int nq = (pp.T + PS::kRows - 1) / PS::kRows;
    PrefillPlan pl = prefill_plan(pp.T, pp.H, st->sm_count);
    if (pl.chunk_tiles > 0) {
        int rc = ensure_workspace(st, kCounterBytes + prefill_partial_bytes(pl, pp.H, D), s);
        if (rc == FR_ERR_WORKSPACE) {
            pl = PrefillPlan();
            pl.units_per_head = nq;
        } else if (rc != FR_OK) {
            return rc;
        }
    }
    if (pl.chunk_tiles > 0) {
        const size_t slots = (size_t)pp.H * pl.slots_per_head;
        pp.chunk_tiles = pl.chunk_tiles;
        pp.slots_per_head = pl.slots_per_head;
        pp.counters = static_cast<int*>(st->ws);
        pp.part_acc = reinterpret_cast<float*>(static_cast<char*>(st->ws) + kCounterBytes);
        pp.part_ml = pp.part_acc + slots * 128 * D;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pp.H, pl.units_per_head, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = PS::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = s != nullptr ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, pp);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

// FORGERT_PREFILL_KERNEL selects the prefill kernel per call: "tc"
// (tcgen05, the default) or "mma" (mma.sync).
bool prefill_use_tc() {
    const char* v = std::getenv("FORGERT_PREFILL_KERNEL");
    return !(v && std::strcmp(v, "mma") == 0);
}

DecodeParams base_params(const void* q, int num_heads, int num_kv_heads) {
    DecodeParams p;
    std::memset(&p, 0, sizeof(p));
    p.q = static_cast<const __half*>(q);
    p.H = num_heads;
    p.Hkv = num_kv_heads;
    p.G = num_heads / num_kv_heads;
    return p;
}

int encode_pair(DecodeParams* p, const void* k, const void* v, int head_dim, int num_kv_heads,
                long long rows) {
    int rc = encode_kv_map(&p->kmap, k, head_dim, num_kv_heads, rows);
    if (rc != FR_OK) return rc;
    return encode_kv_map(&p->vmap, v, head_dim, num_kv_heads, rows);
}

}  // namespace

int* noalloc_error_word(int dev);   // defined with the allocation-free entry point

extern "C" {

int fr_decode_attn(const void* q, const void* k_cache, const void* v_cache, void* out,
                   int num_heads, int num_kv_heads, int head_dim, int kv_len, void* stream) {
    if (!q || !k_cache || !v_cache || !out || kv_len <= 0) return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 4) || !aligned(out, 4))
        return FR_ERR_MISALIGNED;
    DecodeParams p = base_params(q, num_heads, num_kv_heads);
    rc = encode_pair(&p, k_cache, v_cache, head_dim, num_kv_heads, kv_len);
    if (rc != FR_OK) return rc;
    p.kv_len = kv_len;
    // Launch overlap: every row but the newest was written before the
    // preceding kernel ran, so it may stream in before the dependency wait.
    if (g_overlap.load(std::memory_order_relaxed) && stream) p.prefetch_rows = kv_len - 1;
    return run_decode(p, head_dim, 1, kv_len, static_cast<__half*>(out), nullptr, nullptr, 1,
                      static_cast<cudaStream_t>(stream));
}

int fr_decode_attn_batched(const void* q, const void* k_pool, const void* v_pool,
                           const long long* row_offsets, const int* kv_lens, void* out, int batch,
                           int num_heads, int num_kv_heads, int head_dim, long long pool_rows,
                           int max_kv_len, void* stream) {
    if (!q || !k_pool || !v_pool || !row_offsets || !kv_lens || !out || batch <= 0 ||
        max_kv_len < 0 || pool_rows <= 0)
        return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if (!aligned(q, 4) || !aligned(out, 4) || !aligned(k_pool, 16) || !aligned(v_pool, 16) ||
        !aligned(row_offsets, 8) || !aligned(kv_lens, 4))
        return FR_ERR_MISALIGNED;
    DecodeParams p = base_params(q, num_heads, num_kv_heads);
    rc = encode_pair(&p, k_pool, v_pool, head_dim, num_kv_heads, pool_rows);
    if (rc != FR_OK) return rc;
    p.row_offsets = row_offsets;
    p.kv_lens = kv_lens;
    p.zero_tail = 1;
    if (persistent_fits(batch, num_kv_heads, num_heads / num_kv_heads, std::max(1, max_kv_len)))
        return run_persistent(p, head_dim, batch, std::max(1, max_kv_len),
                              static_cast<__half*>(out), static_cast<cudaStream_t>(stream));
    return run_decode(p, head_dim, batch, std::max(1, max_kv_len), static_cast<__half*>(out),
                      nullptr, nullptr, batch_waves(), static_cast<cudaStream_t>(stream));
}

int fr_decode_attn_paged(const void* q, const void* k_pages, const void* v_pages,
                         const int* block_table, const int* kv_lens, void* out, int batch,
                         int num_heads, int num_kv_heads, int head_dim, int page_size,
                         int num_pages, int max_blocks_per_seq, int max_kv_len, void* stream) {
    if (!q || !k_pages || !v_pages || !block_table || !kv_lens || !out || batch <= 0 ||
        num_pages <= 0 || max_blocks_per_seq <= 0 || max_kv_len < 0 || page_size <= 0 ||
        page_size % 16 != 0 || (long long)max_blocks_per_seq * page_size < max_kv_len ||
        (long long)num_pages * page_size >= (1LL << 31))
        return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if (!aligned(q, 4) || !aligned(out, 4) || !aligned(k_pages, 16) || !aligned(v_pages, 16) ||
        !aligned(block_table, 4) || !aligned(kv_lens, 4))
        return FR_ERR_MISALIGNED;
    DecodeParams p = base_params(q, num_heads, num_kv_heads);
    const int box = std::gcd(page_size, tile_rows());    // a box never straddles a page
    const long long rows = (long long)num_pages * page_size;
    rc = encode_kv_map(&p.kmap, k_pages, head_dim, num_kv_heads, rows, box);
    if (rc == FR_OK) rc = encode_kv_map(&p.vmap, v_pages, head_dim, num_kv_heads, rows, box);
    if (rc != FR_OK) return rc;
    p.block_table = block_table;
    p.bt_stride = max_blocks_per_seq;
    p.page_size = page_size;
    p.page_box = box;
    p.num_pages = num_pages;
    p.kv_lens = kv_lens;
    p.zero_tail = 1;        // the last page's rows past the end may hold anything
    return run_decode(p, head_dim, batch, std::max(1, max_kv_len), static_cast<__half*>(out),
                      nullptr, nullptr, batch_waves(), static_cast<cudaStream_t>(stream));
}

int fr_decode_attn_partial(const void* q, const void* k_cache, const void* v_cache, int kv_len,
                           float* state_ml, float* state_acc, int num_heads, int num_kv_heads,
                           int head_dim, void* stream) {
    if (!q || !state_ml || !state_acc || kv_len < 0) return FR_ERR_INVALID_ARG;
    if (kv_len > 0 && (!k_cache || !v_cache)) return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if ((kv_len > 0 && (!aligned(k_cache, 16) || !aligned(v_cache, 16))) || !aligned(q, 4) ||
        !aligned(state_ml, 8) || !aligned(state_acc, 4))
        return FR_ERR_MISALIGNED;
    DecodeParams p = base_params(q, num_heads, num_kv_heads);
    rc = encode_pair(&p, k_cache, v_cache, head_dim, num_kv_heads, kv_len);
    if (rc != FR_OK) return rc;
    p.kv_len = kv_len;
    return run_decode(p, head_dim, 1, std::max(1, kv_len), nullptr, state_ml, state_acc, 1,
                      static_cast<cudaStream_t>(stream));
}

int fr_lse_merge(const float* states_ml, const float* states_acc, int num_states, void* out,
                 int num_heads, int head_dim, void* stream) {
    return fr_lse_merge_strided(states_ml, states_acc, num_states, out, num_heads, head_dim,
                                2LL * num_heads, (long long)num_heads * head_dim, stream);
}

int fr_lse_merge_strided(const float* states_ml, const float* states_acc, int num_states,
                         void* out, int num_heads, int head_dim, long long ml_state_stride,
                         long long acc_state_stride, void* stream) {
    if (!states_ml || !states_acc || !out || num_states <= 0 || num_heads <= 0 ||
        ml_state_stride < 0 || acc_state_stride < 0)
        return FR_ERR_INVALID_ARG;
    if (head_dim != 64 && head_dim != 128) return FR_ERR_UNSUPPORTED;
    if (!aligned(out, 2) || !aligned(states_ml, 8) || !aligned(states_acc, 4) ||
        (ml_state_stride & 1))
        return FR_ERR_MISALIGNED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __half* o = static_cast<__half*>(out);
    const fr::MergeStrides ms{2, ml_state_stride, head_dim, acc_state_stride};
    return head_dim == 64
               ? launch_merge<64>(states_ml, states_acc, num_states, ms, num_heads, o, nullptr,
                                  nullptr, 0, s)
               : launch_merge<128>(states_ml, states_acc, num_states, ms, num_heads, o, nullptr,
                                   nullptr, 0, s);
}

size_t fr_exchange_bytes(int num_heads, int head_dim, int world) {
    if (num_heads <= 0 || (head_dim != 64 && head_dim != 128) || world <= 0 ||
        world > fr::kMaxRanks)
        return 0;
    return fr::XLayout::bytes(world, num_heads, head_dim);
}

int fr_exchange_alloc(size_t bytes, void** buf, void* ipc_handle) {
    if (!buf || !ipc_handle || bytes < fr::XLayout::kHeader) return FR_ERR_INVALID_ARG;
    *buf = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e);
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    *buf = p;
    return FR_OK;
}

int fr_exchange_open(const void* ipc_handle, void** peer_buf) {
    if (!ipc_handle || !peer_buf) return FR_ERR_INVALID_ARG;
    *peer_buf = nullptr;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e);
    *peer_buf = p;
    return FR_OK;
}

int fr_exchange_close(void* peer_buf) {
    if (!peer_buf) return FR_ERR_INVALID_ARG;
    cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

int fr_exchange_free(void* buf) {
    if (!buf) return FR_ERR_INVALID_ARG;
    cudaError_t e = cudaFree(buf);
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

// Zeroes the whole buffer: the epoch restarts at 0, so words tagged by the
// calls before the reset must not survive it.
int fr_exchange_reset(void* buf, size_t bytes, void* stream) {
    if (!buf || bytes < fr::XLayout::kHeader) return FR_ERR_INVALID_ARG;
    cudaError_t e = cudaMemsetAsync(buf, 0, bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

// FORGERT_EXCHANGE_WAIT_MS (read once): how long the exchange waits for the
// other ranks' words, 1 ms .. 5 s, default 1 s.  A longer spin would hold a
// shared GPU busy for no purpose once a peer is gone.
int fr_exchange_wait_limit_ms(void) {
    static const int v = std::min(5000, std::max(1, env_int("FORGERT_EXCHANGE_WAIT_MS", 1000)));
    return v;
}

int fr_decode_attn_exchange(const void* q, const void* k_local, const void* v_local,
                            int local_kv_len, void* out, int num_heads, int num_kv_heads,
                            int head_dim, void* const* bufs, int rank, int world, void* stream) {
    if (!q || !out || !bufs || local_kv_len < 0 || world <= 0 || world > fr::kMaxRanks ||
        rank < 0 || rank >= world)
        return FR_ERR_INVALID_ARG;
    if (local_kv_len > 0 && (!k_local || !v_local)) return FR_ERR_INVALID_ARG;
    for (int j = 0; j < world; ++j)
        if (!bufs[j]) return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if ((local_kv_len > 0 && (!aligned(k_local, 16) || !aligned(v_local, 16))) ||
        !aligned(q, 4) || !aligned(out, 4))
        return FR_ERR_MISALIGNED;
    for (int j = 0; j < world; ++j)
        if (!aligned(bufs[j], 256)) return FR_ERR_MISALIGNED;
    DecodeParams p = base_params(q, num_heads, num_kv_heads);
    rc = encode_pair(&p, k_local, v_local, head_dim, num_kv_heads, local_kv_len);
    if (rc != FR_OK) return rc;
    p.kv_len = local_kv_len;
    for (int j = 0; j < world; ++j) p.xbuf[j] = bufs[j];
    p.xrank = rank;
    p.xworld = world;
    p.xrows = num_heads;
    p.xwait_ms = fr_exchange_wait_limit_ms();
    return run_decode(p, head_dim, 1, std::max(1, local_kv_len), static_cast<__half*>(out),
                      nullptr, nullptr, 1, static_cast<cudaStream_t>(stream));
}

int fr_rope_tables(float* cos_tab, float* sin_tab, int max_seq_len, int head_dim, float base,
                   float scale) {
    if (!cos_tab || !sin_tab || max_seq_len <= 0 || head_dim <= 0 || (head_dim & 1) ||
        !(base > 0.f) || !(scale > 0.f))
        return FR_ERR_INVALID_ARG;
    const int half_d = head_dim / 2;
    std::vector<float> c((size_t)max_seq_len * half_d), s((size_t)max_seq_len * half_d);
    for (int f = 0; f < half_d; ++f) {
        const double inv = 1.0 / (std::pow((double)base, 2.0 * f / (double)head_dim) * (double)scale);
        for (int pos = 0; pos < max_seq_len; ++pos) {
            const double th = (double)pos * inv;
            c[(size_t)pos * half_d + f] = (float)std::cos(th);
            s[(size_t)pos * half_d + f] = (float)std::sin(th);
        }
    }
    cudaError_t e = cudaMemcpy(cos_tab, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaMemcpy(sin_tab, s.data(), s.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e);
    return FR_OK;
}

int fr_rope_tables_device(float* cos_tab, float* sin_tab, int max_seq_len, int head_dim,
                          float base, float scale, void* stream) {
    if (!cos_tab || !sin_tab || max_seq_len <= 0 || head_dim <= 0 || (head_dim & 1) ||
        !(base > 0.f) || !(scale > 0.f))
        return FR_ERR_INVALID_ARG;
    const long long n = (long long)max_seq_len * (head_dim / 2);
    if (n >= (1LL << 31)) return FR_ERR_INVALID_ARG;
    const int threads = 256;
    fr::rope_tables_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0,
                             static_cast<cudaStream_t>(stream)>>>(cos_tab, sin_tab, max_seq_len,
                                                                  head_dim, base, scale);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

int fr_qkv_bias_rope_append(void* q, void* k, void* v, const void* q_bias, const void* k_bias,
                            const void* v_bias, void* k_cache, void* v_cache,
                            const float* cos_tab, const float* sin_tab, int seq_len,
                            int num_heads, int num_kv_heads, int head_dim, int pos_offset,
                            void* stream) {
    if (!q || !k || !v || !k_cache || !v_cache || !cos_tab || !sin_tab || seq_len <= 0 ||
        pos_offset < 0)
        return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if (!aligned(v, 16) || !aligned(v_cache, 16) || !aligned(q, 2) || !aligned(k, 2) ||
        !aligned(k_cache, 2) || !aligned(v_bias, 16) || !aligned(q_bias, 2) ||
        !aligned(k_bias, 2))
        return FR_ERR_MISALIGNED;
    const dim3 grid(seq_len, (fr::rope_items(num_heads, num_kv_heads, head_dim) +
                              fr::kRopeThreads - 1) / fr::kRopeThreads);
    fr::rope_append_kernel<<<grid, fr::kRopeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__half*>(q), static_cast<__half*>(k), static_cast<__half*>(v),
        static_cast<const __half*>(q_bias), static_cast<const __half*>(k_bias),
        static_cast<const __half*>(v_bias), static_cast<__half*>(k_cache),
        static_cast<__half*>(v_cache), cos_tab, sin_tab, num_heads, num_kv_heads, head_dim,
        pos_offset);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return FR_OK;
}

// Without biases v is only read (the kernel writes v back only when biasing it).
int fr_rope_append(void* q, void* k, const void* v, void* k_cache, void* v_cache,
                   const float* cos_tab, const float* sin_tab, int seq_len, int num_heads,
                   int num_kv_heads, int head_dim, int pos_offset, void* stream) {
    return fr_qkv_bias_rope_append(q, k, const_cast<void*>(v), nullptr, nullptr, nullptr,
                                   k_cache, v_cache, cos_tab, sin_tab, seq_len, num_heads,
                                   num_kv_heads, head_dim, pos_offset, stream);
}

int fr_prefill_attn(const void* q, const void* k, const void* v, void* out, int seq_len,
                    int num_heads, int num_kv_heads, int head_dim, void* stream) {
    if (!q || !k || !v || !out || seq_len <= 0) return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if (!aligned(k, 16) || !aligned(v, 16) || !aligned(q, 16) || !aligned(out, 4))
        return FR_ERR_MISALIGNED;
    DeviceState* st = nullptr;
    rc = get_state(&st);
    if (rc != FR_OK) return rc;
    fr::PrefillParams pp;
    std::memset(&pp, 0, sizeof(pp));
    rc = encode_kv_map(&pp.qmap, q, head_dim, num_heads, seq_len);
    if (rc == FR_OK) rc = encode_kv_map(&pp.kmap, k, head_dim, num_kv_heads, seq_len);
    if (rc == FR_OK) rc = encode_kv_map(&pp.vmap, v, head_dim, num_kv_heads, seq_len);
    if (rc != FR_OK) return rc;
    pp.out = static_cast<__half*>(out);
    pp.T = seq_len;
    pp.H = num_heads;
    pp.Hkv = num_kv_heads;
    pp.G = num_heads / num_kv_heads;
    pp.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
    pp.err = st->err;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (prefill_use_tc())
        return head_dim == 64 ? launch_prefill_tc<64>(st, pp, s) : launch_prefill_tc<128>(st, pp, s);
    return head_dim == 64 ? launch_prefill<64>(st, pp, s) : launch_prefill<128>(st, pp, s);
}

int fr_reserve_workspace(size_t bytes) {
    DeviceState* st = nullptr;
    int rc = get_state(&st);
    if (rc != FR_OK) return rc;
    return ensure_workspace(st, bytes, nullptr);
}

size_t fr_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                int max_kv_len) {
    if (batch <= 0 || check_heads(num_heads, num_kv_heads, head_dim) != FR_OK) return 0;
    DeviceState* st = nullptr;
    if (get_state(&st) != FR_OK) return 0;
    const int group = num_heads / num_kv_heads;
    Plan pl1, pl4;
    if (plan_for(st, head_dim, batch, num_kv_heads, group, std::max(1, max_kv_len), 1, &pl1) !=
            FR_OK ||
        plan_for(st, head_dim, batch, num_kv_heads, group, std::max(1, max_kv_len), 4, &pl4) !=
            FR_OK)
        return 0;
    const int splits = std::max(pl1.num_splits, pl4.num_splits) + kClusterCtas;
    size_t need = kCounterBytes + partial_bytes((long long)batch * num_heads, splits, head_dim);
    if (persistent_fits(batch, num_kv_heads, group, std::max(1, max_kv_len))) {
        PersistPlan pp;
        if (persistent_plan(st, head_dim, batch, num_kv_heads, group, std::max(1, max_kv_len),
                            &pp) != FR_OK)
            return 0;
        need = std::max(need, pp.ws_bytes);
    }
    return need;
}

size_t fr_prefill_workspace_size(int seq_len, int num_heads, int head_dim) {
    if (seq_len <= 0 || num_heads <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
    DeviceState* st = nullptr;
    if (get_state(&st) != FR_OK) return 0;
    const PrefillPlan pl = prefill_plan(seq_len, num_heads, st->sm_count);
    return pl.chunk_tiles > 0 ? kCounterBytes + prefill_partial_bytes(pl, num_heads, head_dim) : 0;
}

int fr_get_device_error(int clear, int* device_code) {
    // Reads (and optionally clears) the error words of the current device:
    // the one of the regular entry points and the allocation-free one.  It
    // creates no per-device state and allocates nothing, so callers of
    // fr_decode_attn_noalloc can use it too.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e);
    DeviceState* st = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_dev.find(dev);
        if (it != g_dev.end() && it->second.err) st = &it->second;
    }
    int* words[2] = {st ? st->err : nullptr, noalloc_error_word(dev)};
    int code = 0;
    for (int* w : words) {
        if (!w) continue;
        int c = 0;
        e = cudaMemcpy(&c, w, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_fail(e);
        if (!code) code = c;
        if (clear && c) {
            e = cudaMemset(w, 0, sizeof(int));
            if (e != cudaSuccess) return cuda_fail(e);
        }
    }
    if (clear && code && st && st->ws) {
        // an aborted call may have left fused-merge counters behind
        e = cudaMemset(st->ws, 0, std::min(st->ws_bytes, kCounterBytes));
        if (e != cudaSuccess) return cuda_fail(e);
    }
    if (device_code) *device_code = code;
    return code ? FR_ERR_TIMEOUT : FR_OK;
}

size_t fr_allocated_bytes(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_dev.find(dev);
    if (it == g_dev.end() || !it->second.err) return 0;
    return sizeof(int) + it->second.ws_bytes;
}

int fr_last_cuda_error(void) { return t_last_cuda; }

const char* fr_status_string(int status) {
    switch (status) {
        case FR_OK: return "ok";
        case FR_ERR_INVALID_ARG: return "invalid argument";
        case FR_ERR_UNSUPPORTED: return "unsupported head_dim (64 or 128)";
        case FR_ERR_MISALIGNED: return "misaligned pointer";
        case FR_ERR_CUDA: return "CUDA runtime error";
        case FR_ERR_TIMEOUT: return "in-kernel wait timed out";
        case FR_ERR_WORKSPACE: return "workspace too small during stream capture";
        case FR_ERR_SCRATCH_LIMIT:
            return "problem needs more split scratch than the static no-alloc buffer holds "
                   "(FR_NOALLOC_SCRATCH_BYTES)";
        default: return "unknown status";
    }
}

int fr_version(void) { return kVersion; }

int fr_set_launch_overlap(int enable) { return g_overlap.exchange(enable ? 1 : 0); }

namespace {

// Device-visible address of `p`: device or managed memory as is, page-locked
// host memory through its mapping; nullptr for memory the device cannot reach
// (pageable host memory).
const void* device_view(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    switch (a.type) {
        case cudaMemoryTypeDevice:
        case cudaMemoryTypeManaged:
            return p;
        case cudaMemoryTypeHost:
            return a.devicePointer;
        default:
            return nullptr;
    }
}

}  // namespace

int fr_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
    if (bytes == 0) return FR_OK;
    if (!dst || !src) return FR_ERR_INVALID_ARG;
    const void* s = device_view(src);
    void* d = const_cast<void*>(device_view(dst));
    if (!s || !d) return FR_ERR_INVALID_ARG;
    DeviceState* st = nullptr;
    int rc = get_state(&st);
    if (rc != FR_OK) return rc;
    const bool vec = aligned(s, 16) && aligned(d, 16);
    const size_t units = vec ? bytes / 16 : bytes;
    const size_t per_cta = (size_t)fr::kCopyThreads * fr::kCopyUnroll;
    const size_t ctas = std::max<size_t>(1, std::min<size_t>(2 * (size_t)st->sm_count,
                                                             (units + per_cta - 1) / per_cta));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas, 1, 1);
    cfg.blockDim = dim3(fr::kCopyThreads, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = stream != nullptr ? 1 : 0;
    cudaError_t e;
    if (vec)
        e = cudaLaunchKernelEx(&cfg, fr::copy_kernel, static_cast<const uint4*>(s),
                               static_cast<uint4*>(d), units, (int)(bytes % 16));
    else
        e = cudaLaunchKernelEx(&cfg, fr::copy_bytes_kernel, static_cast<const unsigned char*>(s),
                               static_cast<unsigned char*>(d), units);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}

unsigned long long fr_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

#ifdef FR_TRACE
// Trace builds only (libforgert_b200_trace.so): attach a zeroed device
// buffer of kTraceMaxCtas x kTracePerCta fr::TraceRec records (nullptr
// detaches).  Every record whose time is non-zero is an event.
FR_API int fr_trace_attach(void* buf) {
    cudaError_t e = cudaMemcpyToSymbol(fr::fr_trace_buf, &buf, sizeof(buf));
    return e == cudaSuccess ? FR_OK : cuda_fail(e);
}
#endif

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode (fr_decode_attn_noalloc).
//
// Some callers cannot call cudaMalloc at all: code running inside another
// framework's memory pool or allocator hooks, plugins loaded where the host
// owns every device allocation, or a process that must not grow its device
// footprint after start-up.  For them the split partial states live in this
// file-scope device array instead of the grown-on-demand workspace, and the
// in-kernel error word beside it replaces the cudaMalloc'd one.  Every GPU
// that loads the library holds these FR_NOALLOC_SCRATCH_BYTES (+ 4 bytes)
// until the process exits.
//
// Host code must not use the arrays' names as device addresses (on the host
// they are only stand-in symbols): the set-up below asks the runtime for the
// real addresses with cudaGetSymbolAddress, once per device, with that device
// current, and passes those pointers to the kernels.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char fr_noalloc_scratch[FR_NOALLOC_SCRATCH_BYTES];
static __device__ int fr_noalloc_err;

namespace {

struct NoAllocDevice {
    bool ready = false;
    DeviceState st;              // sm_count / kernel attributes; st.err unused
    float* scratch = nullptr;    // device address of fr_noalloc_scratch on this device
    int* err = nullptr;          // device address of fr_noalloc_err on this device
};

std::mutex g_noalloc_mu;
std::unordered_map<int, NoAllocDevice> g_noalloc;

// First call on a device: symbol addresses, SM count, kernel attributes.  No
// allocation anywhere (cudaGetSymbolAddress, cudaDeviceGetAttribute,
// cudaFuncSetAttribute and the occupancy query allocate nothing).  The
// caller holds g_noalloc_mu.
int noalloc_setup_locked(int dev, NoAllocDevice** out) {
    NoAllocDevice& nd = g_noalloc[dev];
    if (!nd.ready) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, fr_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e);
        void* eptr = nullptr;
        e = cudaGetSymbolAddress(&eptr, fr_noalloc_err);
        if (e != cudaSuccess) return cuda_fail(e);
        e = cudaDeviceGetAttribute(&nd.st.sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e);
        nd.scratch = static_cast<float*>(ptr);
        nd.err = static_cast<int*>(eptr);
        nd.ready = true;
    }
    *out = &nd;
    return FR_OK;
}

}  // namespace

// The no-alloc error word of device `dev` (nullptr when no allocation-free
// call ran there); read by fr_get_device_error.
int* noalloc_error_word(int dev) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    auto it = g_noalloc.find(dev);
    return (it != g_noalloc.end() && it->second.ready) ? it->second.err : nullptr;
}

extern "C" int fr_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                      void* out, int num_heads, int num_kv_heads, int head_dim,
                                      int kv_len, void* stream) {
    if (!q || !k_cache || !v_cache || !out || kv_len <= 0) return FR_ERR_INVALID_ARG;
    int rc = check_heads(num_heads, num_kv_heads, head_dim);
    if (rc != FR_OK) return rc;
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 4) || !aligned(out, 4))
        return FR_ERR_MISALIGNED;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    NoAllocDevice* nd = nullptr;
    const int group = num_heads / num_kv_heads;
    Plan pl;
    {
        // Set-up and planning (which sets kernel attributes and caches the
        // occupancy on first use) under one lock: two host threads making
        // their first call on a device do not race on those fields.
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        rc = noalloc_setup_locked(dev, &nd);
        if (rc != FR_OK) return rc;
        rc = plan_for(&nd->st, head_dim, 1, num_kv_heads, group, kv_len, 1, &pl);
        if (rc != FR_OK) return rc;
    }
    // fr_decode_attn's base split count (one CTA slot per SM) without its
    // cluster sizing or fused merge; a plan whose partials do not fit is
    // refused before anything is launched.
    if (pl.num_splits > 1 &&
        partial_bytes(num_heads, pl.num_splits, head_dim) > (size_t)FR_NOALLOC_SCRATCH_BYTES)
        return FR_ERR_SCRATCH_LIMIT;
    DecodeParams p = base_params(q, num_heads, num_kv_heads);
    rc = encode_pair(&p, k_cache, v_cache, head_dim, num_kv_heads, kv_len);
    if (rc != FR_OK) return rc;
    p.kv_len = kv_len;
    p.G = group;
    p.split_len = pl.split_len;
    p.num_splits = pl.num_splits;
    p.head_groups = pl.head_groups;
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
    p.err = nd->err;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __half* o = static_cast<__half*>(out);
    const bool direct = pl.num_splits == 1;
    if (direct) {
        p.write_final = 1;
        p.out = o;
    } else {
        // Every CTA overwrites its own partial slot (with the neutral state
        // if its bounded wait ran out), so nothing in the scratch needs
        // clearing between calls.
        p.write_final = 0;
        p.part_ml = nd->scratch;
        p.part_acc = nd->scratch + (size_t)num_heads * pl.num_splits * 2;
    }
    p.part_slots = pl.num_splits;
    dim3 grid(p.Hkv * pl.head_groups, pl.num_splits, 1);
    rc = head_dim == 64 ? launch_split_any<64>(p, pl.nt, 1, grid, s, false)
                        : launch_split_any<128>(p, pl.nt, 1, grid, s, false);
    if (rc != FR_OK || direct) return rc;
    const fr::MergeStrides ms{2LL * pl.num_splits, 2, (long long)pl.num_splits * head_dim,
                              head_dim};
    return head_dim == 64 ? launch_merge<64>(p.part_ml, p.part_acc, pl.num_splits, ms, num_heads, o,
                                             nullptr, nullptr, 0, s)
                          : launch_merge<128>(p.part_ml, p.part_acc, pl.num_splits, ms, num_heads,
                                              o, nullptr, nullptr, 0, s);
}
