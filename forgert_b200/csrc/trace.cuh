// trace.cuh - per-CTA phase timestamps for the decode kernels (diagnostics).
//
// Built only into the trace variant of the library (-DFR_TRACE,
// `python -m forgert_b200.build --trace` -> libforgert_b200_trace.so); in
// the product library every FR_TRACE_EV(...) compiles to nothing.
//
// Each CTA index owns kTracePerCta record slots and two counters: how many
// launches it has started (its launch ordinal, fixed at the kEvStart event
// and kept in shared memory for the CTA's later events) and how many records
// it has written.  A record holds the %globaltimer value (ns), the launch
// ordinal, the event id and the SM, so launches that overlap in time (the
// next layer's CTAs start while this layer's still run) stay apart.  The
// host attaches a buffer with fr_trace_attach (trace builds only);
// forgert_b200/phase_trace.py turns the records into per-phase times.
#pragma once
#include <cstdint>

namespace fr {

enum TraceEvent : unsigned {
    kEvStart = 1,        // kernel entry (every CTA; thread 0)
    kEvMeta = 2,         // lengths scanned / partition known (persistent kernel)
    kEvFirstIssue = 3,   // producer issued its first tile
    kEvDepWait = 4,      // consumers past the grid-dependency wait
    kEvQLoaded = 5,      // q fragments in registers
    kEvFirstFull = 6,    // first tile landed (consumer warp 0)
    kEvLoopEnd = 7,      // last tile consumed (consumer warp 0; per item in the persistent kernel)
    kEvFold = 8,         // cross-warp state folded
    kEvStored = 9,       // output or piece stored (per item)
    kEvMergeEnd = 10,    // merge of pieces / clusters done
    kEvXMergeEnd = 11,   // cross-cluster merge (split kernel, last CTA per rank) done
    kEvEnd = 12,         // consumers done
};

constexpr int kTraceMaxCtas = 2048;
constexpr int kTracePerCta = 4096;

struct TraceRec {
    unsigned long long t;
    unsigned launch;     // launch ordinal of this CTA index
    unsigned ev_sm;      // event | sm << 8
};

#ifdef FR_TRACE
__device__ TraceRec* fr_trace_buf = nullptr;          // [kTraceMaxCtas][kTracePerCta]
__device__ unsigned fr_trace_launch[kTraceMaxCtas];
__device__ unsigned fr_trace_fill[kTraceMaxCtas];

__device__ __forceinline__ void trace_event(unsigned ev) {
    __shared__ unsigned s_launch;
    TraceRec* buf = fr_trace_buf;
    if (!buf) return;
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (cta >= kTraceMaxCtas) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    if (ev == kEvStart) s_launch = atomicAdd(&fr_trace_launch[cta], 1u);
    const unsigned k = s_launch;
    const unsigned i = atomicAdd(&fr_trace_fill[cta], 1u);
    if (i < kTracePerCta) buf[(size_t)cta * kTracePerCta + i] = TraceRec{t, k, ev | (sm << 8)};
}
#define FR_TRACE_EV(ev) ::fr::trace_event(ev)
#else
#define FR_TRACE_EV(ev) ((void)0)
#endif

}  // namespace fr
