// Degree reordering on the GPU (replaces sortCSRByDegreeDPLCPU,
// main.cpp:197-278 of the reference, which sorts on the host with oneDPL).
//
// The reference orders rows by (degree ascending, original id ascending), a
// strict total order.  A STABLE sort of the row ids 0..n-1 keyed by degree
// produces exactly that order, so the permutation here is bit-identical:
//   1. keys = degrees, values = row ids (iota);
//   2. LSD radix sort, 8 bits per pass, as many passes as the largest degree
//      needs.  Each pass: per-tile digit histograms, one exclusive scan over
//      the digit-major histogram table, then a stable scatter in which every
//      tile ranks its items with warp match/ballot and per-warp digit counts.
//      A tile is 256 x R items, R in [1, 16] chosen so that a pass has about
//      two tiles per SM (short row arrays would otherwise run on a few CTAs);
//   3. new offsets = exclusive scan of the sorted degrees (int32, since
//      nnz < 2^31 is a precondition of the int32 CSR);
//   4. rows are gathered by output position: each CTA owns 2048 consecutive
//      output nonzeros.  A kernel over rows first records, per chunk, the rows
//      holding its first and last position; the CTA stages the offsets of the
//      (at most 2048) rows in between in shared memory and binary-searches
//      there, so hub rows are split across CTAs and stores are coalesced.  All
//      of a thread's loads are issued before its stores.
// The reference's own GPU sorter (src/utils.cpp:106-339) uses an atomic
// bucket scatter whose tie order is nondeterministic; it is not the parity
// target.
#include <algorithm>

#include "common.cuh"
#include "scan.cuh"

namespace cwlb {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortMaxRounds = 16;  // tile = kSortThreads x rounds items
constexpr int kRadix = 256;

__global__ void degrees_kernel(const int32_t* __restrict__ rowoff, int32_t n, int32_t nnz,
                               uint32_t* __restrict__ keys, int32_t* __restrict__ vals,
                               unsigned int* __restrict__ max_deg, uint32_t* err) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    uint32_t d = 0;
    if (i < n) {
        const int32_t b0 = rowoff[i], b1 = rowoff[i + 1];
        if (b1 < b0 || b0 < 0 || b1 > nnz) atomicOr(err, CWLB_DEVERR_OFFSETS);
        d = b1 > b0 ? static_cast<uint32_t>(b1 - b0) : 0u;
        keys[i] = d;
        vals[i] = static_cast<int32_t>(i);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d = max(d, __shfl_xor_sync(0xffffffffu, d, o));
    if ((threadIdx.x & 31) == 0) atomicMax(max_deg, d);
}

__global__ void __launch_bounds__(kSortThreads)
    radix_hist_kernel(const uint32_t* __restrict__ keys, int32_t n, int shift, int rounds,
                      int64_t n_tiles, int32_t* __restrict__ hist) {
    __shared__ int32_t h[kRadix];
    h[threadIdx.x] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kSortThreads * rounds;
#pragma unroll 4
    for (int r = 0; r < rounds; ++r) {
        const int64_t i = base + r * kSortThreads + threadIdx.x;
        if (i < n) atomicAdd(&h[(keys[i] >> shift) & 0xffu], 1);
    }
    __syncthreads();
    hist[static_cast<int64_t>(threadIdx.x) * n_tiles + blockIdx.x] = h[threadIdx.x];
}

__global__ void __launch_bounds__(kSortThreads)
    radix_scatter_kernel(const uint32_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
                         int32_t n, int shift, int rounds, int64_t n_tiles,
                         const int32_t* __restrict__ offsets, uint32_t* __restrict__ keys_out,
                         int32_t* __restrict__ vals_out) {
    constexpr int kWarps = kSortThreads / 32;
    __shared__ int32_t running[kRadix];
    __shared__ int32_t wcount[kWarps][kRadix + 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    running[threadIdx.x] = offsets[static_cast<int64_t>(threadIdx.x) * n_tiles + blockIdx.x];
    for (int w = 0; w < kWarps; ++w) wcount[w][threadIdx.x] = 0;
    if (threadIdx.x < kWarps) wcount[threadIdx.x][kRadix] = 0;
    __syncthreads();
    const unsigned lt_mask = (1u << lane) - 1u;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kSortThreads * rounds;
    for (int r = 0; r < rounds; ++r) {
        const int64_t i = base + r * kSortThreads + threadIdx.x;
        const bool valid = i < n;
        uint32_t key = 0;
        int32_t v = 0;
        int d = kRadix;  // sentinel digit for items past the end
        if (valid) {
            key = keys_in[i];
            v = vals_in[i];
            d = static_cast<int>((key >> shift) & 0xffu);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int rank = __popc(peers & lt_mask);
        if (rank == 0) wcount[warp][d] = __popc(peers);
        __syncthreads();
        if (valid) {
            int32_t pos = running[d] + rank;
            for (int w = 0; w < warp; ++w) pos += wcount[w][d];
            keys_out[pos] = key;
            vals_out[pos] = v;
        }
        __syncthreads();
        int32_t add = 0;
        for (int w = 0; w < kWarps; ++w) {
            add += wcount[w][threadIdx.x];
            wcount[w][threadIdx.x] = 0;
        }
        running[threadIdx.x] += add;
        __syncthreads();
    }
}

constexpr int kGatherThreads = 256;
constexpr int kGatherItems = 8;
constexpr int kGatherChunk = kGatherThreads * kGatherItems;  // output nnz per CTA

__device__ __forceinline__ int32_t upper_bound_i32(const int32_t* a, int32_t n, int32_t x) {
    int32_t lo = 0, hi = n;
    while (lo < hi) {
        const int32_t mid = lo + ((hi - lo) >> 1);
        if (a[mid] <= x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Rows holding the first and the last position of every output chunk:
// first_row[m] is the row containing m*kGatherChunk, last_row[m] the row
// containing min((m+1)*kGatherChunk, nnz) - 1.  One thread per row writes the
// entries of the chunk boundaries that fall inside it; entries nobody writes
// keep the -1 they were cleared to (only with corrupt offsets).
__global__ void chunk_rows_kernel(const int32_t* __restrict__ new_rowoff, int32_t n, int32_t nnz,
                                  int32_t* __restrict__ first_row, int32_t* __restrict__ last_row,
                                  uint32_t* err) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= n) return;
    const int32_t a = new_rowoff[r], b = new_rowoff[r + 1];
    if (a < 0 || b < a || b > nnz) {
        atomicOr(err, CWLB_DEVERR_OFFSETS);
        return;
    }
    if (a == b) return;
    constexpr int64_t C = kGatherChunk;
    const int64_t n_chunks = (static_cast<int64_t>(nnz) + C - 1) / C;
    // Chunk starts m*C in [a, b).
    for (int64_t m = (a + C - 1) / C; m * C < b; ++m) first_row[m] = static_cast<int32_t>(r);
    // Chunk ends (m+1)*C - 1 in [a, b), i.e. (m+1)*C in [a+1, b].
    for (int64_t m1 = (a + C) / C; m1 * C <= b; ++m1)
        last_row[m1 - 1] = static_cast<int32_t>(r);
    if (b == nnz) last_row[n_chunks - 1] = static_cast<int32_t>(r);  // ragged last chunk
}

__global__ void __launch_bounds__(kGatherThreads)
    gather_rows_kernel(const int32_t* __restrict__ rowoff, const int32_t* __restrict__ col,
                       const float* __restrict__ val, const int32_t* __restrict__ origin,
                       const int32_t* __restrict__ new_rowoff, const int32_t* __restrict__ first_row,
                       const int32_t* __restrict__ last_row, int32_t n, int32_t nnz,
                       int32_t* __restrict__ new_col, float* __restrict__ new_val, uint32_t* err) {
    __shared__ int32_t s_off[kGatherChunk + 1];  // new offsets of the spanned rows
    __shared__ int32_t s_src[kGatherChunk];      // their source offsets
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kGatherChunk;
    const int32_t c1 = static_cast<int32_t>(min(c0 + kGatherChunk, static_cast<int64_t>(nnz)));
    const int32_t r0 = first_row[blockIdx.x];
    const int32_t r1 = last_row[blockIdx.x];
    // Uniform over the CTA: every thread leaves here or none does.
    if (r0 < 0 || r1 < r0 || r1 >= n || r1 - r0 + 1 > kGatherChunk) {
        if (threadIdx.x == 0) atomicOr(err, CWLB_DEVERR_OFFSETS);
        return;
    }
    const int32_t nr = r1 - r0 + 1;
    for (int k = threadIdx.x; k <= nr; k += kGatherThreads) s_off[k] = new_rowoff[r0 + k];
    for (int k = threadIdx.x; k < nr; k += kGatherThreads) s_src[k] = rowoff[origin[r0 + k]];
    __syncthreads();
    int32_t src[kGatherItems];
#pragma unroll
    for (int e = 0; e < kGatherItems; ++e) {
        const int32_t p = static_cast<int32_t>(c0) + e * kGatherThreads + threadIdx.x;
        src[e] = -1;
        if (p < c1) {
            const int32_t k = upper_bound_i32(s_off, nr + 1, p) - 1;
            src[e] = (k >= 0 && k < nr) ? s_src[k] + (p - s_off[k]) : -1;
            if (src[e] < 0 || src[e] >= nnz) {  // only reachable with corrupt offsets
                atomicOr(err, CWLB_DEVERR_OFFSETS);
                src[e] = -1;
            }
        }
    }
    int32_t cv[kGatherItems];
    float vv[kGatherItems];
#pragma unroll
    for (int e = 0; e < kGatherItems; ++e) {
        if (src[e] >= 0) {
            cv[e] = __ldcs(col + src[e]);
            vv[e] = __ldcs(val + src[e]);
        }
    }
#pragma unroll
    for (int e = 0; e < kGatherItems; ++e) {
        if (src[e] >= 0) {
            const int32_t p = static_cast<int32_t>(c0) + e * kGatherThreads + threadIdx.x;
            new_col[p] = cv[e];
            new_val[p] = vv[e];
        }
    }
}

}  // namespace

size_t radix_sort_pairs_scratch_bytes(int32_t n, int sm_count) {
    const int64_t nn = n > 0 ? n : 1;
    const int rounds = static_cast<int>(std::min<int64_t>(
        kSortMaxRounds,
        std::max<int64_t>(1, ceil_div(nn, int64_t{kSortThreads} * 2 * sm_count))));
    const int64_t n_tiles = ceil_div(nn, int64_t{kSortThreads} * rounds);
    auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    return al(sizeof(uint32_t) * nn) + al(sizeof(int32_t) * nn) +
           al(sizeof(int32_t) * n_tiles * kRadix) +
           al(scan_scratch_bytes<int32_t>(n_tiles * kRadix));
}

void radix_sort_pairs(cwlb_ctx* ctx, uint32_t* keys, int32_t* vals, int32_t n, int bits,
                      void* scratch) {
    if (n <= 1 || bits <= 0) return;
    cudaStream_t s = ctx->stream;
    const int sm = ctx->props.multiProcessorCount;
    const int rounds = static_cast<int>(std::min<int64_t>(
        kSortMaxRounds, std::max<int64_t>(1, ceil_div(n, int64_t{kSortThreads} * 2 * sm))));
    const int64_t n_tiles = ceil_div(n, int64_t{kSortThreads} * rounds);
    const int64_t hist_n = n_tiles * kRadix;
    auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    char* p = static_cast<char*>(scratch);
    uint32_t* keys_b = reinterpret_cast<uint32_t*>(p);
    int32_t* vals_b = reinterpret_cast<int32_t*>(p + al(sizeof(uint32_t) * n));
    int32_t* hist = reinterpret_cast<int32_t*>(p + al(sizeof(uint32_t) * n) + al(sizeof(int32_t) * n));
    void* scan_tmp = p + al(sizeof(uint32_t) * n) + al(sizeof(int32_t) * n) +
                     al(sizeof(int32_t) * hist_n);
    uint32_t* kin = keys;
    uint32_t* kout = keys_b;
    int32_t* vin = vals;
    int32_t* vout = vals_b;
    const int passes = (bits + 7) / 8;
    for (int pass = 0; pass < passes; ++pass) {
        const int shift = 8 * pass;
        radix_hist_kernel<<<static_cast<unsigned>(n_tiles), kSortThreads, 0, s>>>(
            kin, n, shift, rounds, n_tiles, hist);
        CWLB_LAUNCH_CHECK("radix_hist_kernel");
        device_exclusive_scan<int32_t>(hist, hist, hist_n, scan_tmp, s);
        radix_scatter_kernel<<<static_cast<unsigned>(n_tiles), kSortThreads, 0, s>>>(
            kin, vin, n, shift, rounds, n_tiles, hist, kout, vout);
        CWLB_LAUNCH_CHECK("radix_scatter_kernel");
        std::swap(kin, kout);
        std::swap(vin, vout);
    }
    if (kin != keys) {
        CWLB_CUDA(cudaMemcpyAsync(keys, kin, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s));
        CWLB_CUDA(cudaMemcpyAsync(vals, vin, sizeof(int32_t) * n, cudaMemcpyDeviceToDevice, s));
    }
}

void launch_sort_by_degree(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                           const int32_t* col, const float* val, int32_t* origin,
                           int32_t* new_rowoff, int32_t* new_col, float* new_val) {
    if (n_rows <= 0) return;
    cudaStream_t s = ctx->stream;
    const int64_t n = n_rows;
    // About two tiles per SM per pass, 256..4096 items per tile.
    const int rounds = static_cast<int>(std::min<int64_t>(
        kSortMaxRounds,
        std::max<int64_t>(1, ceil_div(n, int64_t{kSortThreads} * 2 *
                                             ctx->props.multiProcessorCount))));
    const int64_t n_tiles = ceil_div(n, int64_t{kSortThreads} * rounds);
    const int64_t hist_n = n_tiles * kRadix;
    const int64_t n_chunks = ceil_div(nnz, kGatherChunk);
    // Scratch layout (256-byte aligned pieces).
    auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    const size_t b_keys = al(sizeof(uint32_t) * (n + 1));
    const size_t b_vals = al(sizeof(int32_t) * n);
    const size_t b_hist = al(sizeof(int32_t) * hist_n);
    const size_t b_scan = al(std::max(scan_scratch_bytes<int32_t>(hist_n),
                                      scan_scratch_bytes<int32_t>(n + 1)));
    const size_t b_chunk = al(sizeof(int32_t) * std::max<int64_t>(n_chunks, 1));
    char* p = static_cast<char*>(
        ctx->sort_scratch.ensure(2 * b_keys + b_vals + b_hist + b_scan + 256 + 2 * b_chunk));
    uint32_t* keys_a = reinterpret_cast<uint32_t*>(p);
    uint32_t* keys_b = reinterpret_cast<uint32_t*>(p + b_keys);
    int32_t* vals_b = reinterpret_cast<int32_t*>(p + 2 * b_keys);
    int32_t* hist = reinterpret_cast<int32_t*>(p + 2 * b_keys + b_vals);
    void* scan_tmp = p + 2 * b_keys + b_vals + b_hist;
    unsigned int* d_max = reinterpret_cast<unsigned int*>(p + 2 * b_keys + b_vals + b_hist + b_scan);
    int32_t* first_row = reinterpret_cast<int32_t*>(p + 2 * b_keys + b_vals + b_hist + b_scan + 256);
    int32_t* last_row = first_row + b_chunk / sizeof(int32_t);
    int32_t* vals_a = origin;  // ping-pong through the caller's output

    CWLB_CUDA(cudaMemsetAsync(d_max, 0, sizeof(unsigned int), s));
    degrees_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(
        rowoff, n_rows, nnz, keys_a, vals_a, d_max, ctx->d_error_flags);
    CWLB_LAUNCH_CHECK("degrees_kernel");
    unsigned int max_deg = 0;
    CWLB_CUDA(cudaMemcpyAsync(&max_deg, d_max, sizeof(max_deg), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    int passes = 0;
    while (passes < 4 && (max_deg >> (8 * passes)) != 0u) ++passes;

    uint32_t* kin = keys_a;
    uint32_t* kout = keys_b;
    int32_t* vin = vals_a;
    int32_t* vout = vals_b;
    for (int pass = 0; pass < passes; ++pass) {
        const int shift = 8 * pass;
        radix_hist_kernel<<<static_cast<unsigned>(n_tiles), kSortThreads, 0, s>>>(
            kin, n_rows, shift, rounds, n_tiles, hist);
        CWLB_LAUNCH_CHECK("radix_hist_kernel");
        device_exclusive_scan<int32_t>(hist, hist, hist_n, scan_tmp, s);
        radix_scatter_kernel<<<static_cast<unsigned>(n_tiles), kSortThreads, 0, s>>>(
            kin, vin, n_rows, shift, rounds, n_tiles, hist, kout, vout);
        CWLB_LAUNCH_CHECK("radix_scatter_kernel");
        std::swap(kin, kout);
        std::swap(vin, vout);
    }
    if (vin != origin) {
        CWLB_CUDA(cudaMemcpyAsync(origin, vin, sizeof(int32_t) * n, cudaMemcpyDeviceToDevice, s));
    }
    // New offsets: exclusive scan over the n sorted degrees plus a trailing 0.
    CWLB_CUDA(cudaMemsetAsync(kin + n, 0, sizeof(uint32_t), s));
    device_exclusive_scan<int32_t>(reinterpret_cast<const int32_t*>(kin), new_rowoff, n + 1,
                                   scan_tmp, s);
    if (nnz > 0) {
        CWLB_CUDA(cudaMemsetAsync(first_row, 0xff, 2 * b_chunk, s));  // -1: no row yet
        chunk_rows_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(
            new_rowoff, n_rows, nnz, first_row, last_row, ctx->d_error_flags);
        CWLB_LAUNCH_CHECK("chunk_rows_kernel");
        gather_rows_kernel<<<static_cast<unsigned>(n_chunks), kGatherThreads, 0, s>>>(
            rowoff, col, val, origin, new_rowoff, first_row, last_row, n_rows, nnz, new_col,
            new_val, ctx->d_error_flags);
        CWLB_LAUNCH_CHECK("gather_rows_kernel");
    }
}

}  // namespace cwlb
