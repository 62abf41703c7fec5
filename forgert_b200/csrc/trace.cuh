// trace.cuh - per-CTA phase timestamps for the decode kernels (diagnostics).
//
// Built only into the trace variant of the library (-DFR_TRACE,
// `python -m forgert_b200.build --trace` -> libforgert_b200_trace.so); in
// the product library every FR_TRACE_EV(...) compiles to nothing.
//
// A record holds the %globaltimer value (ns), the low 32 bits of the grid's
// launch number (%gridid, unique per launch in a context), the event id and
// the SM, so launches that overlap in time (the next layer's CTAs start
// while this layer's still run) stay apart.  Recording costs a timer read,
// a shared-memory increment and one store that nobody waits for - no
// global atomics, whose round trips would stretch the phases being timed.
// Each CTA index owns kTraceLaunches blocks of kTraceEvents records; a
// launch writes block (gridid mod kTraceLaunches), so the last
// kTraceLaunches launches of a kernel stay apart.  All events come from
// thread 0 except the producer's kEvFirstIssue, which takes the block's last
// record.  The host zeroes the buffer and attaches it with fr_trace_attach
// (trace builds only); forgert_b200/phase_trace.py reads every record whose
// time is non-zero.
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
    kEvCounted = 13,     // pieces counted after the range (persistent kernel)
    kEvMergeBegin = 14,  // a unit's merge starts (persistent kernel)
    kEvMergeLoaded = 15, // the merge's first loads have landed (persistent kernel)
    kEvFoldSynced = 16,  // consumer warps past their last tile (split kernel)
    kEvStateDone = 17,   // CTA state complete, whole CTA synchronised (split kernel)
    kEvClusterReady = 18,// cluster barrier passed, pushes start (split kernel)
    kEvRecvDone = 19,    // every cluster rank's message received (split kernel)
    kEvFoldStored = 20,  // thread 0's accumulator fragments stored for the fold (split kernel)
    kEvFoldWeights = 21, // per-warp fold weights known (split kernel)
};

constexpr int kTraceMaxCtas = 2048;
constexpr int kTraceLaunches = 128;
constexpr int kTraceEvents = 32;
constexpr int kTracePerCta = kTraceLaunches * kTraceEvents;

struct TraceRec {
    unsigned long long t;
    unsigned launch;     // low 32 bits of %gridid
    unsigned ev_sm;      // event | sm << 8
};

#ifdef FR_TRACE
__constant__ TraceRec* fr_trace_buf = nullptr;        // [kTraceMaxCtas][kTraceLaunches][kTraceEvents]

__device__ __forceinline__ void trace_event(unsigned ev) {
    __shared__ unsigned s_n;                         // thread 0's records in this launch
    TraceRec* buf = fr_trace_buf;
    if (!buf) return;
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (cta >= kTraceMaxCtas) return;
    unsigned long long t, gid;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    asm volatile("mov.u64 %0, %%gridid;" : "=l"(gid));
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    unsigned i;
    if (ev == kEvFirstIssue) {
        i = kTraceEvents - 1;
    } else {
        if (ev == kEvStart) s_n = 0;
        i = s_n;
        if (i >= kTraceEvents - 1) return;
        s_n = i + 1;
    }
    const size_t blk = (size_t)cta * kTraceLaunches + (size_t)(gid % kTraceLaunches);
    buf[blk * kTraceEvents + i] = TraceRec{t, (unsigned)gid, ev | (sm << 8)};
}
#define FR_TRACE_EV(ev) ::fr::trace_event(ev)
#else
#define FR_TRACE_EV(ev) ((void)0)
#endif

}  // namespace fr
