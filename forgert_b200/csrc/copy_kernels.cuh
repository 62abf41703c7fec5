// copy_kernels.cuh - stream-ordered copies by a kernel (fr_copy_async).
//
// The per-step host transfers of a decode step are small (one layer's q is
// H*D*2 bytes, a token id or an argmax result a few bytes).  Through the copy
// engine each such cudaMemcpyAsync costs ~10 us on B200 whatever its size and
// ends the programmatic overlap of the kernels around it.  Page-locked host
// memory is mapped into the device's address space, so a kernel can move
// those bytes itself: every thread keeps kCopyUnroll 16-byte loads in flight
// over the host link, and the kernel takes part in programmatic dependent
// launch like the attention kernels (the next kernel may start its own
// pre-wait work while the copy runs).
#pragma once
#include <cstddef>
#include <cstdint>
#include "fr_ptx.cuh"

namespace fr {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;

// Copies n16 16-byte vectors (both pointers 16-byte aligned), then `tail`
// single bytes after them.
__global__ void __launch_bounds__(kCopyThreads)
copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n16, int tail) {
    grid_launch_dependents();
    grid_dependency_wait();                   // src may come from the preceding grid
    const size_t stride = (size_t)gridDim.x * kCopyThreads;
    size_t i = (size_t)blockIdx.x * kCopyThreads + threadIdx.x;
    for (; i + (kCopyUnroll - 1) * stride < n16; i += kCopyUnroll * stride) {
        uint4 v[kCopyUnroll];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) v[u] = src[i + u * stride];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) dst[i + u * stride] = v[u];
    }
    for (; i < n16; i += stride) dst[i] = src[i];
    if (blockIdx.x == 0 && threadIdx.x < tail) {
        const unsigned char* s = reinterpret_cast<const unsigned char*>(src + n16);
        unsigned char* d = reinterpret_cast<unsigned char*>(dst + n16);
        d[threadIdx.x] = s[threadIdx.x];
    }
}

// Unaligned pointers: byte copy.
__global__ void __launch_bounds__(kCopyThreads)
copy_bytes_kernel(const unsigned char* __restrict__ src, unsigned char* __restrict__ dst,
                  size_t n) {
    grid_launch_dependents();
    grid_dependency_wait();
    const size_t stride = (size_t)gridDim.x * kCopyThreads;
    for (size_t i = (size_t)blockIdx.x * kCopyThreads + threadIdx.x; i < n; i += stride)
        dst[i] = src[i];
}

}  // namespace fr
