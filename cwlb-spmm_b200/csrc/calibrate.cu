// Operation-cost calibration on the B200 (replaces measure_spmm_costs,
// src/utils.cpp:342-829 of the reference, which the costWrite program runs).
//
// Four microbenchmarks, each with 20 untimed launches and `repeat` timed
// launches measured with CUDA events; each result is normalised exactly as the
// reference normalises it (nanoseconds per operation, times 10):
//   compute : WI threads, each a chain of K dependent FMAs acc = fma(acc, a, b)
//             -> C_compute = (mean ms * 1e6 / WI) / K * 10         (:370-427)
//   load    : WI threads in 32-lane groups; each group reads one random K-float
//             row of a data_MB_for_load MiB array, lane l reading columns
//             l, l+32, ... (wrapped mod K)
//             -> C_load = (mean ms * 1e6 / WI) / K * 10            (:429-531)
//   store   : WI threads each write K floats, consecutive threads adjacent
//             -> C_store = (mean ms * 1e6 / WI) / K * 10           (:533-591)
//   atomic  : 128-thread pseudo groups, `atomic_target_writers` groups per
//             output row, K_block = clamp(floor(min(K,128)/32)*32, 32..128)
//             columns, float atomic add of 1.0
//             -> C_atomic = mean ms * 1e6 / (groups * K_block) * 10 (:593-825)
// The random rows of the load benchmark come from std::mt19937_64(123456789)
// with a uniform_int_distribution over the rows, as in the reference.
#include <algorithm>
#include <random>
#include <vector>

#include "common.cuh"

namespace cwlb {
namespace {

constexpr int kCalWarmup = 20;

__global__ void cal_compute_kernel(float* __restrict__ sink, int WI, int K) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= WI) return;
    float acc = 0.0f;
    const float a = 1.001f, b = 0.999f;
    for (int k = 0; k < K; ++k) acc = fmaf(acc, a, b);
    sink[i] = acc;
}

__global__ void cal_load_kernel(const float* __restrict__ data, const uint32_t* __restrict__ idx,
                                int WI, int K, float* __restrict__ sink) {
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= WI) return;
    const int lane = static_cast<int>(gid % 32);
    const uint32_t row = idx[gid - lane];
    const float* base = data + static_cast<int64_t>(row) * K;
    float s = 0.0f;
    for (int t = 0; t < K; ++t) {
        int k = t * 32 + lane;
        if (k >= K) k %= K;
        s += __ldg(base + k);
    }
    // Keep the loads: the sum is stored only in the impossible case s < -1e30
    // (the array holds 1.2345f), which the compiler cannot prove.
    if (s < -1e30f) sink[gid] = s;
}

__global__ void cal_store_kernel(float* __restrict__ out, int WI, int K) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (tid >= WI) return;
    for (int i = 0; i < K; ++i) out[static_cast<int64_t>(i) * WI + tid] = static_cast<float>(i);
}

__global__ void cal_atomic_kernel(float* __restrict__ counters, int64_t total_threads,
                                  int groups_per_row, int G, int K_block) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total_threads) return;
    const int lane = static_cast<int>(t % 128);
    const int64_t group = t / 128;
    const int64_t row = group / groups_per_row;
    if (row >= G) return;
    for (int kk = lane; kk < K_block; kk += 128) {
        atomicAdd(counters + row * K_block + kk, 1.0f);
    }
}

// Gather ceiling: the aggregation's own access pattern without the sparse
// bookkeeping.  Every group of L lanes reads whole rows of L*P float4s (the
// rows of X at K = 4*L*P features) chosen uniformly at random among 2^row_bits
// rows, with U rows (U*P = 8 float4s per lane) in flight, through the same
// read-only path (__ldg) as the aggregation.  Row numbers are the top bits of
// a per-group linear congruential sequence (x = 1664525 x + 1013904223 mod
// 2^32, the Numerical Recipes constants) seeded by the lowbias32 hash
// (C. Wellons, public domain) of the group id: three instructions a row and
// no index array, so neither instruction issue nor index traffic limits the
// rate.  A buffer that fits in L2 gives the rate for rows served from L2; one
// far larger than L2 the rate for rows served from HBM.
__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

template <int P, int U>
__global__ void __launch_bounds__(256)
    cal_gather_kernel(const float4* __restrict__ buf, int row_bits, int L, int iters,
                      float* __restrict__ sink) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    const int sub = static_cast<int>(tid % static_cast<uint32_t>(L));
    const int64_t row4 = static_cast<int64_t>(L) * P;
    const int shift = 32 - row_bits;  // row_bits in [1, 31]
    uint32_t x = lowbias32(tid / static_cast<uint32_t>(L));
    float s = 0.f;
    for (int it = 0; it < iters; ++it) {
        float4 v[U][P];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            x = x * 1664525u + 1013904223u;
            const float4* q = buf + static_cast<int64_t>(x >> shift) * row4 + sub;
#pragma unroll
            for (int j = 0; j < P; ++j) v[u][j] = __ldg(q + j * L);
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int j = 0; j < P; ++j) s += (v[u][j].x + v[u][j].y) + (v[u][j].z + v[u][j].w);
    }
    // The buffer holds zeros: the store never happens, but the compiler
    // cannot prove it, so the loads stay.
    if (s != 0.f) sink[tid % 1024] = s;
}

template <typename Launch>
double mean_ms(cwlb_ctx* ctx, int repeat, Launch launch) {
    for (int w = 0; w < kCalWarmup; ++w) launch();
    CWLB_LAUNCH_CHECK("calibration warm-up");
    CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
    double total = 0.0;
    for (int r = 0; r < repeat; ++r) {
        CWLB_CUDA(cudaEventRecord(ctx->ev_start, ctx->stream));
        launch();
        CWLB_CUDA(cudaEventRecord(ctx->ev_stop, ctx->stream));
        CWLB_CUDA(cudaEventSynchronize(ctx->ev_stop));
        float ms = 0.0f;
        CWLB_CUDA(cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop));
        total += ms;
    }
    CWLB_LAUNCH_CHECK("calibration launch");
    return total / repeat;
}

struct DevMem {
    void* p = nullptr;
    explicit DevMem(size_t bytes) { CWLB_CUDA(cudaMalloc(&p, bytes < 256 ? 256 : bytes)); }
    ~DevMem() {
        if (p) cudaFree(p);
    }
    template <typename T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

}  // namespace

void measure_costs(cwlb_ctx* ctx, int K, int repeat, int WI, int data_MB, int writers,
                   cwlb_costs* out) {
    cudaStream_t s = ctx->stream;
    const int threads = 256;
    const unsigned blocks = static_cast<unsigned>(ceil_div(WI, threads));
    *out = cwlb_costs{};
    out->K = K;
    out->WI = WI;
    out->repeat = repeat;

    {  // compute
        DevMem sink(sizeof(float) * static_cast<size_t>(WI));
        const double ms = mean_ms(ctx, repeat, [&] {
            cal_compute_kernel<<<blocks, threads, 0, s>>>(sink.as<float>(), WI, K);
        });
        out->C_compute_ns = (ms * 1e6) / static_cast<double>(WI) / static_cast<double>(K) * 10;
    }
    {  // load
        const size_t total_floats = static_cast<size_t>(data_MB) * 1024ull * 1024ull / sizeof(float);
        if (total_floats < static_cast<size_t>(K)) fail(CWLB_ERR_RUNTIME, "data_MB_for_load too small for K.");
        const size_t rows = total_floats / static_cast<size_t>(K);
        DevMem data(sizeof(float) * total_floats);
        DevMem idx(sizeof(uint32_t) * static_cast<size_t>(WI));
        DevMem sink(sizeof(float) * static_cast<size_t>(WI));
        std::vector<float> init(std::min<size_t>(total_floats, size_t(1) << 22), 1.2345f);
        for (size_t off = 0; off < total_floats; off += init.size()) {
            const size_t n = std::min(init.size(), total_floats - off);
            CWLB_CUDA(cudaMemcpy(data.as<float>() + off, init.data(), n * sizeof(float),
                                 cudaMemcpyHostToDevice));
        }
        std::vector<uint32_t> h_idx(static_cast<size_t>(WI));
        std::mt19937_64 rng(123456789ULL);
        std::uniform_int_distribution<uint32_t> dist(0U, static_cast<uint32_t>(rows - 1));
        for (int g = 0; g < WI; g += 32) {
            const uint32_t row = dist(rng);
            for (int t = 0; t < 32 && g + t < WI; ++t) h_idx[g + t] = row;
        }
        CWLB_CUDA(cudaMemcpy(idx.as<uint32_t>(), h_idx.data(), sizeof(uint32_t) * WI,
                             cudaMemcpyHostToDevice));
        const double ms = mean_ms(ctx, repeat, [&] {
            cal_load_kernel<<<blocks, threads, 0, s>>>(data.as<float>(), idx.as<uint32_t>(), WI, K,
                                                       sink.as<float>());
        });
        out->C_load_ns = (ms * 1e6) / static_cast<double>(WI) / static_cast<double>(K) * 10;
    }
    {  // store
        DevMem buf(sizeof(float) * static_cast<size_t>(WI) * static_cast<size_t>(K));
        const double ms = mean_ms(ctx, repeat, [&] {
            cal_store_kernel<<<blocks, threads, 0, s>>>(buf.as<float>(), WI, K);
        });
        out->C_store_ns = (ms * 1e6) / static_cast<double>(WI) / static_cast<double>(K) * 10;
    }
    {  // atomic
        const int groups_per_row = std::max(1, writers);
        int K_block = std::min(K, 128);
        K_block = (K_block / 32) * 32;
        if (K_block <= 0) K_block = 32;
        const int target = std::max(1, (WI + 127) / 128);
        int G = std::max(1, target / groups_per_row);
        while (static_cast<int64_t>(G) * groups_per_row < target) ++G;
        const int64_t total_groups = static_cast<int64_t>(G) * groups_per_row;
        const int64_t total_threads = total_groups * 128;
        const size_t counters_n = static_cast<size_t>(G) * static_cast<size_t>(K_block);
        DevMem counters(sizeof(float) * counters_n);
        const unsigned ab = static_cast<unsigned>(ceil_div(total_threads, threads));
        double total = 0.0;
        for (int w = 0; w < kCalWarmup; ++w) {
            CWLB_CUDA(cudaMemsetAsync(counters.p, 0, sizeof(float) * counters_n, s));
            cal_atomic_kernel<<<ab, threads, 0, s>>>(counters.as<float>(), total_threads,
                                                     groups_per_row, G, K_block);
        }
        CWLB_LAUNCH_CHECK("calibration atomic warm-up");
        for (int r = 0; r < repeat; ++r) {
            CWLB_CUDA(cudaMemsetAsync(counters.p, 0, sizeof(float) * counters_n, s));
            CWLB_CUDA(cudaEventRecord(ctx->ev_start, s));
            cal_atomic_kernel<<<ab, threads, 0, s>>>(counters.as<float>(), total_threads,
                                                     groups_per_row, G, K_block);
            CWLB_CUDA(cudaEventRecord(ctx->ev_stop, s));
            CWLB_CUDA(cudaEventSynchronize(ctx->ev_stop));
            float ms = 0.0f;
            CWLB_CUDA(cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop));
            total += ms;
        }
        CWLB_LAUNCH_CHECK("calibration atomic");
        const double avg_ms = total / repeat;
        const double ops = static_cast<double>(total_groups) * static_cast<double>(K_block);
        out->C_atomic_ns = (avg_ms * 1e6) / ops * 10.0;
        out->atomic_writers_per_addr = groups_per_row;
    }
}

double measure_gather_gbs(cwlb_ctx* ctx, int buffer_MB, int row_floats, int repeat) {
    cudaStream_t s = ctx->stream;
    const int row4 = row_floats / 4;
    // The aggregation's lane shapes: two float4s per lane where the row has
    // at least two (16 lanes x 2 at K = 128, 4 x 2 at K = 32, 32 x 4 at K = 512).
    const int L = std::max(1, std::min(row4 / 2, 32));  // lanes per row
    const int P = row4 / L;                              // float4s per lane per row
    const int64_t row_bytes = int64_t{row4} * 16;
    // A power-of-two number of rows, 2 .. 2^31, at most the buffer's.
    const int64_t fit = static_cast<int64_t>(buffer_MB) * 1024 * 1024 / row_bytes;
    if (fit < 2) fail(CWLB_ERR_INVALID_ARGUMENT, "buffer_MB holds fewer than two rows.");
    int row_bits = 1;
    while (row_bits < 31 && (int64_t{1} << (row_bits + 1)) <= fit) ++row_bits;
    const int64_t rows = int64_t{1} << row_bits;
    DevMem buf(static_cast<size_t>(rows * row_bytes));
    DevMem sink(sizeof(float) * 1024);
    CWLB_CUDA(cudaMemsetAsync(buf.p, 0, static_cast<size_t>(rows * row_bytes), s));
    // Rows in flight per lane group as in the aggregation: U*P = 8 float4s.
    const int U = 8 / P;
    const void* fn = P == 1   ? reinterpret_cast<const void*>(&cal_gather_kernel<1, 8>)
                     : P == 2 ? reinterpret_cast<const void*>(&cal_gather_kernel<2, 4>)
                     : P == 4 ? reinterpret_cast<const void*>(&cal_gather_kernel<4, 2>)
                              : reinterpret_cast<const void*>(&cal_gather_kernel<8, 1>);
    int per_sm = 0;
    CWLB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, 0));
    const unsigned blocks =
        static_cast<unsigned>(ctx->props.multiProcessorCount) * static_cast<unsigned>(std::max(1, per_sm));
    const int64_t groups = int64_t{blocks} * 256 / L;
    // About 4 GB gathered per launch (at least one iteration).
    const int iters = static_cast<int>(std::max<int64_t>(
        1, (int64_t{1} << 32) / (groups * U * row_bytes)));
    auto launch = [&] {
        const float4* b = buf.as<float4>();
        float* k = sink.as<float>();
        switch (P) {
            case 1: cal_gather_kernel<1, 8><<<blocks, 256, 0, s>>>(b, row_bits, L, iters, k); break;
            case 2: cal_gather_kernel<2, 4><<<blocks, 256, 0, s>>>(b, row_bits, L, iters, k); break;
            case 4: cal_gather_kernel<4, 2><<<blocks, 256, 0, s>>>(b, row_bits, L, iters, k); break;
            default: cal_gather_kernel<8, 1><<<blocks, 256, 0, s>>>(b, row_bits, L, iters, k); break;
        }
    };
    const double ms = mean_ms(ctx, repeat, launch);
    const double bytes = static_cast<double>(groups) * iters * U * static_cast<double>(row_bytes);
    return bytes / (ms * 1e-3) / 1e9;
}

}  // namespace cwlb
