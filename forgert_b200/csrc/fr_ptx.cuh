// fr_ptx.cuh - sm_100a device helpers used by the decode-attention kernels.
//
// Thin inline-PTX wrappers for the Blackwell data-movement and tensor paths
// the kernels are built on:
//   * mbarrier phase tracking with expect-tx accounting (bounded waits),
//   * cp.async.bulk / cp.async.bulk.tensor (TMA, global -> this CTA's shared memory),
//   * ldmatrix / movmatrix / mma.sync m16n8k16 (f16 in, f32 accumulate),
//   * ex2.approx for the base-2 online softmax.
// Every wait has a time limit: a wait that runs out records an error code in
// a device word the host reads back, and the kernel returns instead of
// spinning forever.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace fr {

// Error codes written to the device error word (host maps them to status).
enum DeviceError : int {
    kDevOk = 0,
    kDevTimeoutFull = 1,   // consumer gave up waiting for a stage to land
    kDevTimeoutEmpty = 2,  // producer gave up waiting for a stage to drain
    kDevTimeoutPeer = 3,   // cross-GPU exchange: the other ranks' states never all arrived
};

// Wall-clock budget of one bounded wait (ns).  Real waits last microseconds;
// one second means the pipeline is wedged.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(tx) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// The waiting thread is suspended until the phase completes or, at the
// latest, after kSuspendHintNs, so idle warps do not spin on issue slots the
// computing warps need.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs) : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false if
// the wait ran past kWaitLimitNs (the caller records the error and unwinds).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// ------------------------------------------ TMA tensor copy (into this CTA only)
// 4-D tiled load described by a CUtensorMap that lives in kernel parameter
// space (__grid_constant__).  Coordinates are element indices, innermost
// first; out-of-bounds box elements are written as zeros and still count
// towards the transaction bytes.
__device__ __forceinline__ void tma_load_4d(void* dst_smem, const void* tmap, int c0, int c1,
                                            int c2, int c3, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;"
        :: "r"(smem_u32(dst_smem)), "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
           "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Prefetch of one global line into L2 (a hint; nothing is returned).
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" :: "l"(p) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}

// ------------------------------------------- TMA bulk copy (into this CTA only)
// Copies `bytes` (multiple of 16, both addresses 16-byte aligned) from global
// to this CTA's shared memory and signals completion on `bar` as tx bytes.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem,
                                         uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1], %2, [%3];"
        :: "r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 eviction hint: the KV cache is streamed exactly once per
// call, so it is marked evict-first to keep L2 for the partial states.
__device__ __forceinline__ void bulk_g2s_evict_first(void* dst_smem, const void* src_gmem,
                                                     uint32_t bytes, uint64_t* bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;"
        :: "r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// --------------------------------------------------- clusters / DSMEM / PDL
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of all CTAs of the cluster; release/acquire orders shared and
// global accesses around it at cluster scope.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Split form: arrive (release) early, wait (acquire) later, so the barrier is
// off the critical path.
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local_smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// 16-byte store into another CTA's shared memory (cluster address) that
// completes 16 transaction bytes on that CTA's mbarrier (cluster address).
__device__ __forceinline__ void st_async_v4(uint32_t addr, float4 v, uint32_t mbar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
        :: "r"(addr), "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)),
           "r"(__float_as_uint(v.z)), "r"(__float_as_uint(v.w)), "r"(mbar)
        : "memory");
}

__device__ __forceinline__ void st_dsmem_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" :: "r"(addr), "r"(v) : "memory");
}

// Release increment (no value returned): publishes the stores this thread
// has observed (e.g. its warp's, ordered before by __syncwarp).
__device__ __forceinline__ void red_add_release_gpu(int* addr, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" :: "l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* addr) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// Atomic add with acquire-release semantics at GPU scope: orders every write
// this thread has observed (including other threads' writes published to it
// by a barrier) before the add, and the add before later reads.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* addr, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;"
                 : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

// Atomic add with release semantics at GPU scope (orders this thread's
// earlier accesses, and those a barrier ordered before it, before the add).
__device__ __forceinline__ int atom_add_release_gpu(int* addr, int v) {
    int old;
    asm volatile("atom.add.release.gpu.global.s32 %0, [%1], %2;"
                 : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

// Relaxed atomic add at GPU scope (ordering comes from fences around it).
__device__ __forceinline__ int atom_add_relaxed_gpu(int* addr, int v) {
    int old;
    asm volatile("atom.add.relaxed.gpu.global.s32 %0, [%1], %2;"
                 : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

// Acquire-release fence at GPU scope.  Unlike __threadfence() (a
// sequentially consistent fence) it only orders this thread's own accesses:
// before a relaxed atomic it releases, after one it acquires.
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// 8-byte system-scope relaxed store / load.  An aligned 8-byte access is
// single-copy atomic, so a 4-byte value stored together with a 4-byte tag is
// seen by another GPU either whole or not at all: the tag tells the reader
// that the value has arrived (no fence or separate flag needed).
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* addr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* addr) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// Programmatic dependent launch: wait until the grids this one depends on
// have completed and their writes are visible; let the next grid launch.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ tensor-core ops
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// Transposes an 8x8 b16 matrix held in the standard fragment layout
// (lane holds row lane/4, columns 2*(lane%4) and 2*(lane%4)+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 2^x with the hardware approximation (MUFU.EX2); ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace fr
