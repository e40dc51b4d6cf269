// Device-wide exclusive prefix sum (reduce-then-scan, no inter-block waits).
//
// Three phases per level: each block reduces a tile of kScanTile items, the
// tile sums are scanned (recursively when there are more than kScanTile of
// them), and each block rescans its tile seeded with its tile offset.  No
// block ever waits on another, so there is no spin loop to bound.
#pragma once

#include "common.cuh"

namespace cwlb {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;  // 4096

template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* smem_warp, T& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        T w = lane < kScanThreads / 32 ? smem_warp[lane] : T(0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const T y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kScanThreads / 32) smem_warp[lane] = w;
    }
    __syncthreads();
    const T warp_prefix = warp > 0 ? smem_warp[warp - 1] : T(0);
    total = smem_warp[kScanThreads / 32 - 1];
    __syncthreads();
    return warp_prefix + x - v;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads)
    scan_reduce_kernel(const T* __restrict__ in, int64_t n, T* __restrict__ tile_sums) {
    __shared__ T sw[kScanThreads / 32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
    T s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const int64_t idx = base + static_cast<int64_t>(i) * kScanThreads + threadIdx.x;
        if (idx < n) s += in[idx];
    }
    T total;
    block_exclusive_scan<T>(s, sw, total);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// Each thread owns kScanItems consecutive items (blocked layout).  in and out
// may be the same array (no __restrict__ on them): every thread reads all of
// its items before it writes any, and no other thread touches them.
template <typename T>
__global__ void __launch_bounds__(kScanThreads)
    scan_apply_kernel(const T* in, int64_t n, const T* __restrict__ tile_offsets, T* out) {
    __shared__ T sw[kScanThreads / 32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile +
                         static_cast<int64_t>(threadIdx.x) * kScanItems;
    T v[kScanItems];
    T s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        v[i] = (base + i < n) ? in[base + i] : T(0);
        s += v[i];
    }
    T total;
    T run = block_exclusive_scan<T>(s, sw, total) + (tile_offsets ? tile_offsets[blockIdx.x] : T(0));
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        if (base + i < n) out[base + i] = run;
        run += v[i];
    }
}

// Bytes of scratch needed by device_exclusive_scan for n items.
template <typename T>
inline size_t scan_scratch_bytes(int64_t n) {
    size_t bytes = 0;
    int64_t m = n;
    while (m > kScanTile) {
        m = ceil_div(m, kScanTile);
        bytes += 2 * sizeof(T) * static_cast<size_t>(m) + 256;
    }
    return bytes + 256;
}

// out[i] = sum(in[0..i)); in and out may alias.  scratch must hold
// scan_scratch_bytes<T>(n) bytes.
template <typename T>
void device_exclusive_scan(const T* in, T* out, int64_t n, void* scratch, cudaStream_t s) {
    if (n <= 0) return;
    if (n <= kScanTile) {
        scan_apply_kernel<T><<<1, kScanThreads, 0, s>>>(in, n, nullptr, out);
        CWLB_LAUNCH_CHECK("scan_apply_kernel");
        return;
    }
    const int64_t tiles = ceil_div(n, kScanTile);
    T* sums = static_cast<T*>(scratch);
    T* offs = sums + tiles;
    char* rest = reinterpret_cast<char*>(offs + tiles);
    rest += (256 - reinterpret_cast<uintptr_t>(rest) % 256) % 256;
    scan_reduce_kernel<T><<<static_cast<unsigned>(tiles), kScanThreads, 0, s>>>(in, n, sums);
    CWLB_LAUNCH_CHECK("scan_reduce_kernel");
    device_exclusive_scan<T>(sums, offs, tiles, rest, s);
    scan_apply_kernel<T><<<static_cast<unsigned>(tiles), kScanThreads, 0, s>>>(in, n, offs, out);
    CWLB_LAUNCH_CHECK("scan_apply_kernel");
}

}  // namespace cwlb
