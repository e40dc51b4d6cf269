// C ABI of libcwlb_spmm: contexts, error reporting and the host-buffer entry
// points that mirror the reference's synchronous functions.  Every exported
// function converts internal failures into a cwlb_status and a thread-local
// message; no C++ exception crosses the boundary.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <future>
#include <iomanip>
#include <limits>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace {

thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return CWLB_OK;
    } catch (const cwlb::Failure& e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return CWLB_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return CWLB_ERR_RUNTIME;
    }
}

void require(bool ok, int code, const char* msg) {
    if (!ok) cwlb::fail(code, msg);
}

void check_ctx(cwlb_ctx* ctx) {
    require(ctx != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null context");
    CWLB_CUDA(cudaSetDevice(ctx->device));
}

template <typename T>
T* stage_h2d(cwlb_ctx* ctx, cwlb::DeviceBuffer& buf, const T* host, size_t count) {
    T* d = buf.as<T>(count);
    cwlb::copy_to_device(ctx, d, host, sizeof(T) * count, ctx->stream);
    return d;
}

uint32_t take_device_errors(cwlb_ctx* ctx) {
    uint32_t flags = 0;
    CWLB_CUDA(cudaMemcpyAsync(&flags, ctx->d_error_flags, sizeof(flags), cudaMemcpyDeviceToHost,
                              ctx->stream));
    CWLB_CUDA(cudaMemsetAsync(ctx->d_error_flags, 0, sizeof(uint32_t), ctx->stream));
    CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
    return flags;
}

void raise_device_errors(uint32_t flags) {
    if (!flags) return;
    std::string m = "invalid input detected on the device:";
    if (flags & CWLB_DEVERR_COL_RANGE) m += " column index outside [0, H.rows());";
    if (flags & CWLB_DEVERR_ROW_RANGE) m += " task row outside [0, rows);";
    if (flags & CWLB_DEVERR_OFFSETS) m += " row offsets not monotone or beyond nnz;";
    if (flags & CWLB_DEVERR_ORIGIN_RANGE) m += " Origin_local id outside [0, rows);";
    cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, m);
}

// True when every value is exactly 1.0f (the reference's text loader gives
// every stored entry the value 1, src/data.cpp).  Scans with up to 16 host
// threads and stops at the first other value.
bool all_ones(const float* v, size_t n) {
    if (n == 0) return true;
    constexpr uint32_t kOne = 0x3f800000u;
    const size_t per_thread_min = size_t(1) << 20;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const unsigned T = static_cast<unsigned>(
        std::min<size_t>(std::min(16u, hw), (n + per_thread_min - 1) / per_thread_min));
    std::atomic<bool> other{false};
    auto scan = [&](size_t b, size_t e) {
        constexpr size_t kBlock = size_t(1) << 16;
        for (size_t i = b; i < e; i += kBlock) {
            if (other.load(std::memory_order_relaxed)) return;
            const size_t end = std::min(e, i + kBlock);
            uint32_t acc = 0;
            for (size_t j = i; j < end; ++j) {
                uint32_t w;
                std::memcpy(&w, v + j, sizeof(w));
                acc |= w ^ kOne;
            }
            if (acc) {
                other.store(true, std::memory_order_relaxed);
                return;
            }
        }
    };
    if (T <= 1) {
        scan(0, n);
    } else {
        std::vector<std::thread> pool;
        const size_t chunk = (n + T - 1) / T;
        for (unsigned t = 1; t < T; ++t) {
            const size_t b = std::min(n, t * chunk);
            pool.emplace_back(scan, b, std::min(n, b + chunk));
        }
        scan(0, std::min(n, chunk));
        for (auto& th : pool) th.join();
    }
    return !other.load();
}

// Chunked copy plan for a host-buffer call: chunk c holds tasks
// [task_cut[c], task_cut[c+1]) and needs nonzeros [0, nnz_cut[c+1]).  Possible
// when every task's rows are in range and the tasks are in order of their
// last nonzero (as the partitioner emits them); small calls are not split.
bool plan_pipeline(const int32_t* row_offset, int32_t n_rows, int32_t nnz, const cwlb_task* tasks,
                   int64_t n_tasks, int64_t (&task_cut)[cwlb_ctx::kPipeChunks + 1],
                   int64_t (&nnz_cut)[cwlb_ctx::kPipeChunks + 1]) {
    constexpr int C = cwlb_ctx::kPipeChunks;
    if (nnz < (1 << 22) || n_tasks < 8 * C) return false;
    std::vector<int64_t> last(static_cast<size_t>(n_tasks));
    int64_t prev = 0;
    for (int64_t t = 0; t < n_tasks; ++t) {
        const cwlb_task& k = tasks[t];
        if (k.row_start < 0 || k.row_end > n_rows || k.row_start >= k.row_end) return false;
        const int64_t b = row_offset[k.row_end - 1], e = row_offset[k.row_end];
        if (b < 0 || e < b || e > nnz) return false;
        const int64_t end = k.last_row_nnz > 0 ? std::min<int64_t>(e, b + k.last_row_nnz) : e;
        if (end < prev) return false;
        last[static_cast<size_t>(t)] = prev = end;
    }
    task_cut[0] = 0;
    nnz_cut[0] = 0;
    for (int c = 1; c < C; ++c) {
        const int64_t target = static_cast<int64_t>(nnz) * c / C;
        int64_t t = std::upper_bound(last.begin(), last.end(), target) - last.begin();
        t = std::max(t, task_cut[c - 1]);
        task_cut[c] = t;
        nnz_cut[c] = t > 0 ? last[static_cast<size_t>(t - 1)] : 0;
    }
    task_cut[C] = n_tasks;
    nnz_cut[C] = nnz;
    return true;
}

template <typename T>
void copy_h2d(cwlb_ctx* ctx, T* dst, const T* src, int64_t count, cudaStream_t s) {
    if (count > 0) cwlb::copy_to_device(ctx, dst, src, sizeof(T) * static_cast<size_t>(count), s);
}

// Host-buffer aggregation.  All copies go on the context's copy stream: the
// row offsets, origins, tasks and X first, then the column ids in chunks (see
// plan_pipeline; one chunk when the tasks cannot be chunked), then the values
// unless they are all one (checked on the host while the copies run).  The
// compute stream aggregates chunk c's tasks as soon as chunk c has arrived,
// while later chunks are still being copied.  `time_us` is the sum of the
// aggregation kernels' times.
void spmm_host_staged(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                      const int32_t* col_ind, const float* value, const int32_t* origin,
                      const float* H, int64_t h_rows, int64_t K, const cwlb_task* tasks,
                      int64_t n_tasks, float* out, double* time_us) {
    constexpr int C = cwlb_ctx::kPipeChunks;
    cudaStream_t cs = ctx->copy_stream, ks = ctx->stream;
    const size_t out_count = static_cast<size_t>(n_rows) * static_cast<size_t>(K);
    int32_t* d_ro = ctx->in_rowoff.as<int32_t>(static_cast<size_t>(n_rows) + 1);
    int32_t* d_col = ctx->in_col.as<int32_t>(static_cast<size_t>(nnz));
    int32_t* d_org = ctx->in_origin.as<int32_t>(static_cast<size_t>(n_rows));
    float* d_H = ctx->in_H.as<float>(static_cast<size_t>(h_rows) * static_cast<size_t>(K));
    cwlb_task* d_tasks = ctx->in_tasks.as<cwlb_task>(static_cast<size_t>(n_tasks));
    float* d_out = ctx->out_buf.as<float>(out_count);
    bool launched[C] = {};
    int n_chunks = 1;
    try {
        // The values are checked on other host threads while this one queues
        // (or, for pageable memory, stages) the copies.
        std::future<bool> unit = std::async(std::launch::async, all_ones, value,
                                            static_cast<size_t>(nnz));
        // Copies start after whatever the compute stream has queued.
        CWLB_CUDA(cudaEventRecord(ctx->ev_start, ks));
        CWLB_CUDA(cudaStreamWaitEvent(cs, ctx->ev_start, 0));
        copy_h2d(ctx, d_ro, row_offset, static_cast<int64_t>(n_rows) + 1, cs);
        copy_h2d(ctx, d_org, origin, n_rows, cs);
        copy_h2d(ctx, d_tasks, tasks, n_tasks, cs);
        copy_h2d(ctx, d_H, H, h_rows * K, cs);
        int64_t task_cut[C + 1] = {0, n_tasks}, nnz_cut[C + 1] = {0, nnz};
        if (plan_pipeline(row_offset, n_rows, nnz, tasks, n_tasks, task_cut, nnz_cut)) n_chunks = C;
        for (int c = 0; c < n_chunks; ++c) {
            copy_h2d(ctx, d_col + nnz_cut[c], col_ind + nnz_cut[c], nnz_cut[c + 1] - nnz_cut[c], cs);
            CWLB_CUDA(cudaEventRecord(ctx->pipe_ready[c], cs));
        }
        const float* d_val = nullptr;  // all values 1.0: the kernels read none
        if (!unit.get()) {
            float* dv = ctx->in_val.as<float>(static_cast<size_t>(nnz));
            for (int c = 0; c < n_chunks; ++c) {
                copy_h2d(ctx, dv + nnz_cut[c], value + nnz_cut[c], nnz_cut[c + 1] - nnz_cut[c], cs);
                CWLB_CUDA(cudaEventRecord(ctx->pipe_ready[c], cs));  // now after the values
            }
            d_val = dv;
        }
        if (out_count) CWLB_CUDA(cudaMemsetAsync(d_out, 0, sizeof(float) * out_count, ks));
        for (int c = 0; c < n_chunks; ++c) {
            const int64_t t0 = task_cut[c], nt = task_cut[c + 1] - task_cut[c];
            if (nt <= 0) continue;
            CWLB_CUDA(cudaStreamWaitEvent(ks, ctx->pipe_ready[c], 0));
            CWLB_CUDA(cudaEventRecord(ctx->pipe_t0[c], ks));
            cwlb::launch_spmm_mean(ctx, n_rows, nnz, d_ro, d_col, d_val, d_org, d_H, h_rows, K,
                                   d_tasks + t0, nt, d_out,
                                   cwlb::kFlagOutCleared | cwlb::task_variant_flag(ctx, n_tasks, 0),
                                   nullptr, 0, cwlb::task_run_length(nnz, n_tasks));
            CWLB_CUDA(cudaEventRecord(ctx->pipe_t1[c], ks));
            launched[c] = true;
        }
        cwlb::copy_to_host(ctx, out, d_out, sizeof(float) * out_count, ks);
    } catch (...) {
        // No copy may still read the caller's arrays once the call returns.
        cudaStreamSynchronize(cs);
        cudaStreamSynchronize(ks);
        throw;
    }
    CWLB_CUDA(cudaStreamSynchronize(cs));
    raise_device_errors(take_device_errors(ctx));
    double us = 0.0;
    for (int c = 0; c < n_chunks; ++c) {
        if (!launched[c]) continue;
        float ms = 0.0f;
        CWLB_CUDA(cudaEventElapsedTime(&ms, ctx->pipe_t0[c], ctx->pipe_t1[c]));
        us += static_cast<double>(ms) * 1e3;
    }
    *time_us = us;
}

// Shared body of cwlb_spmm_kernel / cwlb_spmm_kernel_large_k.
void spmm_host(cwlb_ctx* ctx, bool large_k, int32_t n_rows, int32_t nnz,
               const int32_t* row_offset, const int32_t* col_ind, const float* value,
               const int32_t* origin, const float* H, int64_t h_rows, int64_t K,
               int32_t local_dimension, const cwlb_task* tasks, int64_t n_tasks, float* out,
               double* time_us) {
    check_ctx(ctx);
    require(time_us != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null time output");
    require(n_rows >= 0 && nnz >= 0 && h_rows >= 0 && K >= 0 && n_tasks >= 0,
            CWLB_ERR_INVALID_ARGUMENT, "negative size");
    const int64_t max_wg = ctx->props.maxThreadsPerBlock;
    const size_t out_count = static_cast<size_t>(n_rows) * static_cast<size_t>(K);
    if (!large_k) {
        // spmmKernel: K == 0 first, then the work-group limit, then empty tasks
        // (src/parallelMatrix.cpp:80-104).
        if (K == 0) {
            *time_us = 0.0;
            return;
        }
        if (K > max_wg) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT,
                       "spmmKernel supports only K <= device max work-group size; "
                       "use spmmKernelLargeKFallback for larger K.");
        }
    } else {
        // spmmKernelLargeKFallback (src/parallelMatrix.cpp:283-294).
        if (K <= max_wg) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT,
                       "spmmKernelLargeKFallback requires K > device max work-group size.");
        }
    }
    if (n_tasks == 0) {
        if (out_count) std::memset(out, 0, sizeof(float) * out_count);
        *time_us = 0.0;
        return;
    }
    // The reference sizes its local-memory tile from local_dimension; a
    // non-positive tile cannot make progress there, so it is rejected here.
    if (!large_k) {
        require(local_dimension > 0, CWLB_ERR_INVALID_ARGUMENT,
                "local_dimension must be positive");
    }
    require(row_offset && origin && tasks && out && (nnz == 0 || (col_ind && value)) &&
                (h_rows * K == 0 || H),
            CWLB_ERR_INVALID_ARGUMENT, "null input pointer");

    spmm_host_staged(ctx, n_rows, nnz, row_offset, col_ind, value, origin, H, h_rows, K, tasks,
                     n_tasks, out, time_us);
}

cwlb_costs zero_costs() {
    cwlb_costs c{};
    return c;
}

}  // namespace

void cwlb::set_last_error(const std::string& msg) { g_last_error = msg; }

extern "C" {

const char* cwlb_last_error(void) { return g_last_error.c_str(); }

const char* cwlb_version(void) { return "cwlb-spmm-b200 0.1.0 (sm_100a)"; }

int cwlb_ctx_create(int device, cwlb_ctx** out) {
    return guarded([&] {
        require(out != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null output");
        *out = nullptr;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            cwlb::fail(CWLB_ERR_NO_DEVICE, "no CUDA device available");
        }
        require(device >= 0 && device < n, CWLB_ERR_NO_DEVICE, "device index out of range");
        auto* ctx = new cwlb_ctx();
        try {
            ctx->device = device;
            CWLB_CUDA(cudaSetDevice(device));
            CWLB_CUDA(cudaGetDeviceProperties(&ctx->props, device));
            if (ctx->props.major < 10) {
                cwlb::fail(CWLB_ERR_NO_DEVICE,
                           "libcwlb_spmm is built for sm_100a (B200); device " +
                               std::string(ctx->props.name) + " is not compute capability 10.x");
            }
            CWLB_CUDA(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
            ctx->own_stream = true;
            CWLB_CUDA(cudaEventCreate(&ctx->ev_start));
            CWLB_CUDA(cudaEventCreate(&ctx->ev_stop));
            CWLB_CUDA(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking));
            CWLB_CUDA(cudaEventCreateWithFlags(&ctx->plan_fork, cudaEventDisableTiming));
            CWLB_CUDA(cudaEventCreateWithFlags(&ctx->plan_join, cudaEventDisableTiming));
            for (int c = 0; c < cwlb_ctx::kPipeChunks; ++c) {
                CWLB_CUDA(cudaEventCreateWithFlags(&ctx->pipe_ready[c], cudaEventDisableTiming));
                CWLB_CUDA(cudaEventCreate(&ctx->pipe_t0[c]));
                CWLB_CUDA(cudaEventCreate(&ctx->pipe_t1[c]));
            }
            CWLB_CUDA(cudaMalloc(&ctx->d_error_flags, sizeof(uint32_t)));
            CWLB_CUDA(cudaMemset(ctx->d_error_flags, 0, sizeof(uint32_t)));
        } catch (...) {
            cwlb_ctx_destroy(ctx);
            throw;
        }
        *out = ctx;
    });
}

int cwlb_ctx_destroy(cwlb_ctx* ctx) {
    if (!ctx) return CWLB_OK;
    return guarded([&] {
        cudaSetDevice(ctx->device);
        if (ctx->stream) cudaStreamSynchronize(ctx->stream);
        cwlb::destroy_stager(ctx);
        for (cwlb::DeviceBuffer* b : {&ctx->in_rowoff, &ctx->in_col, &ctx->in_val, &ctx->in_origin,
                                      &ctx->in_H, &ctx->in_tasks, &ctx->out_buf, &ctx->sort_scratch,
                                      &ctx->part_scratch, &ctx->part_desc, &ctx->part_tasks,
                                      &ctx->check_scratch, &ctx->det_scratch})
            b->release();
        if (ctx->d_error_flags) cudaFree(ctx->d_error_flags);
        if (ctx->copy_stream) cudaStreamSynchronize(ctx->copy_stream);
        if (ctx->ev_start) cudaEventDestroy(ctx->ev_start);
        if (ctx->plan_fork) cudaEventDestroy(ctx->plan_fork);
        if (ctx->plan_join) cudaEventDestroy(ctx->plan_join);
        if (ctx->ev_stop) cudaEventDestroy(ctx->ev_stop);
        for (int c = 0; c < cwlb_ctx::kPipeChunks; ++c) {
            if (ctx->pipe_ready[c]) cudaEventDestroy(ctx->pipe_ready[c]);
            if (ctx->pipe_t0[c]) cudaEventDestroy(ctx->pipe_t0[c]);
            if (ctx->pipe_t1[c]) cudaEventDestroy(ctx->pipe_t1[c]);
        }
        if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
        if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
    });
}

int cwlb_ctx_set_stream(cwlb_ctx* ctx, void* stream) {
    return guarded([&] {
        check_ctx(ctx);
        if (ctx->own_stream && ctx->stream) {
            CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
            CWLB_CUDA(cudaStreamDestroy(ctx->stream));
        }
        ctx->stream = static_cast<cudaStream_t>(stream);
        ctx->own_stream = false;
    });
}

void* cwlb_ctx_stream(cwlb_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int cwlb_ctx_synchronize(cwlb_ctx* ctx) {
    return guarded([&] {
        check_ctx(ctx);
        CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int cwlb_ctx_take_device_errors(cwlb_ctx* ctx, uint32_t* flags) {
    return guarded([&] {
        check_ctx(ctx);
        require(flags != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null output");
        *flags = take_device_errors(ctx);
    });
}

int cwlb_device_info(cwlb_ctx* ctx, int64_t* max_wg, int32_t* cus, int64_t* local_mem,
                     char* name, size_t name_cap) {
    return guarded([&] {
        check_ctx(ctx);
        if (max_wg) *max_wg = ctx->props.maxThreadsPerBlock;
        if (cus) *cus = ctx->props.multiProcessorCount;
        if (local_mem) *local_mem = static_cast<int64_t>(ctx->props.sharedMemPerBlock);
        if (name && name_cap) {
            std::strncpy(name, ctx->props.name, name_cap - 1);
            name[name_cap - 1] = '\0';
        }
    });
}

int cwlb_spmm_kernel(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                     const int32_t* col_ind, const float* value, const int32_t* origin_local,
                     const float* H, int64_t h_rows, int64_t K, int32_t dim_hint,
                     int32_t local_dimension, const cwlb_task* tasks, int64_t n_tasks,
                     float* out, double* time_us) {
    (void)dim_hint;
    return guarded([&] {
        spmm_host(ctx, false, n_rows, nnz, row_offset, col_ind, value, origin_local, H, h_rows,
                  K, local_dimension, tasks, n_tasks, out, time_us);
    });
}

int cwlb_spmm_kernel_large_k(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                             const int32_t* row_offset, const int32_t* col_ind,
                             const float* value, const int32_t* origin_local, const float* H,
                             int64_t h_rows, int64_t K, int32_t dim_hint,
                             int32_t local_dimension, const cwlb_task* tasks, int64_t n_tasks,
                             float* out, double* time_us) {
    (void)dim_hint;
    return guarded([&] {
        spmm_host(ctx, true, n_rows, nnz, row_offset, col_ind, value, origin_local, H, h_rows,
                  K, local_dimension, tasks, n_tasks, out, time_us);
    });
}

int cwlb_spmm_mean_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                          const int32_t* d_row_offset, const int32_t* d_col_ind,
                          const float* d_value, const int32_t* d_origin_local, const float* d_H,
                          int64_t h_rows, int64_t K, const cwlb_task* d_tasks, int64_t n_tasks,
                          float* d_out, uint32_t flags) {
    return guarded([&] {
        check_ctx(ctx);
        require(n_rows >= 0 && nnz >= 0 && h_rows >= 0 && K >= 0 && n_tasks >= 0,
                CWLB_ERR_INVALID_ARGUMENT, "negative size");
        require((flags & ~static_cast<uint32_t>(CWLB_ROWS_COVERED | CWLB_DETERMINISTIC |
                                                CWLB_TASK_PER_WARP | CWLB_TASK_PER_CTA)) == 0,
                CWLB_ERR_INVALID_ARGUMENT, "unknown flags");
        require((flags & (CWLB_TASK_PER_WARP | CWLB_TASK_PER_CTA)) !=
                    (CWLB_TASK_PER_WARP | CWLB_TASK_PER_CTA),
                CWLB_ERR_INVALID_ARGUMENT, "CWLB_TASK_PER_WARP and CWLB_TASK_PER_CTA exclude each other");
        cwlb::launch_spmm_mean(ctx, n_rows, nnz, d_row_offset, d_col_ind, d_value,
                               d_origin_local, d_H, h_rows, K, d_tasks, n_tasks, d_out, flags);
    });
}

int cwlb_spmm_mean_reference_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                                    const int32_t* d_row_offset, const int32_t* d_col_ind,
                                    const float* d_value, const float* d_H, int64_t h_rows,
                                    int64_t K, float* d_out) {
    return guarded([&] {
        check_ctx(ctx);
        require(n_rows >= 0 && nnz >= 0 && h_rows >= 0 && K >= 0, CWLB_ERR_INVALID_ARGUMENT,
                "negative size");
        cwlb::launch_spmm_mean_reference(ctx, n_rows, nnz, d_row_offset, d_col_ind, d_value, d_H,
                                         h_rows, K, d_out);
    });
}

int cwlb_tasks_check(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* d_row_offset,
                     const cwlb_task* d_tasks, int64_t n_tasks, int64_t* bad_tasks,
                     int64_t* uncovered_rows, int64_t* nnz_coverage_errors) {
    return guarded([&] {
        check_ctx(ctx);
        require(bad_tasks && uncovered_rows && nnz_coverage_errors, CWLB_ERR_INVALID_ARGUMENT,
                "null output");
        cwlb::run_tasks_check(ctx, n_rows, nnz, d_row_offset, d_tasks, n_tasks, bad_tasks,
                              uncovered_rows, nnz_coverage_errors);
    });
}

int cwlb_sort_by_degree(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                        const int32_t* col_ind, const float* value, int32_t* origin_local,
                        int32_t* sorted_row_offset, int32_t* sorted_col_ind,
                        float* sorted_value) {
    return guarded([&] {
        check_ctx(ctx);
        require(n_rows >= 0 && nnz >= 0, CWLB_ERR_INVALID_ARGUMENT, "negative size");
        if (n_rows == 0) return;  // the reference returns an empty CSR_Order
        require(row_offset[n_rows] == nnz, CWLB_ERR_RUNTIME,
                "DPL CPU degree reordering produced an inconsistent NNZ count.");
        const int32_t* d_ro = stage_h2d(ctx, ctx->in_rowoff, row_offset, static_cast<size_t>(n_rows) + 1);
        const int32_t* d_col = stage_h2d(ctx, ctx->in_col, col_ind, static_cast<size_t>(nnz));
        const float* d_val = stage_h2d(ctx, ctx->in_val, value, static_cast<size_t>(nnz));
        // Outputs staged in out_buf: origin | offsets | cols | values.
        const size_t n = static_cast<size_t>(n_rows);
        char* o = static_cast<char*>(ctx->out_buf.ensure(4 * (n + n + 1) + 8 * static_cast<size_t>(nnz) + 64));
        int32_t* d_org = reinterpret_cast<int32_t*>(o);
        int32_t* d_nro = d_org + n;
        int32_t* d_ncol = d_nro + n + 1;
        float* d_nval = reinterpret_cast<float*>(d_ncol + nnz);
        cwlb::launch_sort_by_degree(ctx, n_rows, nnz, d_ro, d_col, d_val, d_org, d_nro, d_ncol, d_nval);
        cudaStream_t s = ctx->stream;
        cwlb::copy_to_host(ctx, origin_local, d_org, 4 * n, s);
        cwlb::copy_to_host(ctx, sorted_row_offset, d_nro, 4 * (n + 1), s);
        cwlb::copy_to_host(ctx, sorted_col_ind, d_ncol, 4 * static_cast<size_t>(nnz), s);
        cwlb::copy_to_host(ctx, sorted_value, d_nval, 4 * static_cast<size_t>(nnz), s);
        require(sorted_row_offset[n_rows] == nnz, CWLB_ERR_RUNTIME,
                "DPL CPU degree reordering produced an inconsistent NNZ count.");
    });
}

int cwlb_sort_by_degree_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                               const int32_t* d_row_offset, const int32_t* d_col_ind,
                               const float* d_value, int32_t* d_origin_local,
                               int32_t* d_sorted_row_offset, int32_t* d_sorted_col_ind,
                               float* d_sorted_value) {
    return guarded([&] {
        check_ctx(ctx);
        require(n_rows >= 0 && nnz >= 0, CWLB_ERR_INVALID_ARGUMENT, "negative size");
        if (n_rows == 0) return;
        cwlb::launch_sort_by_degree(ctx, n_rows, nnz, d_row_offset, d_col_ind, d_value,
                                    d_origin_local, d_sorted_row_offset, d_sorted_col_ind,
                                    d_sorted_value);
    });
}

int cwlb_partition(cwlb_ctx* ctx, int32_t n_rows, const int32_t* row_offset,
                   const cwlb_costs* costs, double capacity, cwlb_task* tasks,
                   int64_t max_tasks, int64_t* n_tasks) {
    return guarded([&] {
        check_ctx(ctx);
        require(costs && n_tasks, CWLB_ERR_INVALID_ARGUMENT, "null argument");
        *n_tasks = 0;
        if (n_rows <= 0) return;
        const int32_t* d_ro = stage_h2d(ctx, ctx->in_rowoff, row_offset, static_cast<size_t>(n_rows) + 1);
        const int64_t cnt = cwlb::run_partition(ctx, n_rows, d_ro, *costs, capacity);
        *n_tasks = cnt;
        if (!tasks) return;
        if (max_tasks < cnt) {
            cwlb::fail(CWLB_ERR_BUFFER_TOO_SMALL, "task buffer too small");
        }
        cwlb::copy_to_host(ctx, tasks, ctx->part_tasks.ptr, sizeof(cwlb_task) * cnt, ctx->stream);
        CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int cwlb_partition_device(cwlb_ctx* ctx, int32_t n_rows, const int32_t* d_row_offset,
                          const cwlb_costs* costs, double capacity, cwlb_task** d_tasks,
                          int64_t* n_tasks) {
    return guarded([&] {
        check_ctx(ctx);
        require(costs && d_tasks && n_tasks, CWLB_ERR_INVALID_ARGUMENT, "null argument");
        *n_tasks = 0;
        *d_tasks = nullptr;
        if (n_rows <= 0) return;
        *n_tasks = cwlb::run_partition(ctx, n_rows, d_row_offset, *costs, capacity);
        *d_tasks = static_cast<cwlb_task*>(ctx->part_tasks.ptr);
    });
}

int cwlb_measure_spmm_costs(cwlb_ctx* ctx, int32_t K, int32_t repeat, int32_t WI,
                            int32_t data_MB_for_load, int32_t atomic_target_writers,
                            cwlb_costs* out) {
    return guarded([&] {
        check_ctx(ctx);
        require(out != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null output");
        if (K <= 0 || repeat <= 0 || WI <= 0 || data_MB_for_load <= 0 || atomic_target_writers <= 0) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "All microbenchmark parameters must be positive.");
        }
        cwlb::measure_costs(ctx, K, repeat, WI, data_MB_for_load, atomic_target_writers, out);
    });
}

int cwlb_measure_gather_gbs(cwlb_ctx* ctx, int32_t buffer_MB, int32_t row_floats,
                            int32_t repeat, double* gbs) {
    return guarded([&] {
        check_ctx(ctx);
        require(gbs != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null output");
        if (buffer_MB <= 0 || repeat <= 0) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "All microbenchmark parameters must be positive.");
        }
        const int32_t row4 = row_floats / 4;
        if (row_floats <= 0 || row_floats % 4 != 0 || row4 > 256 || (row4 & (row4 - 1)) != 0) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT,
                       "row_floats must be 4 times a power of two, at most 1024.");
        }
        *gbs = cwlb::measure_gather_gbs(ctx, buffer_MB, row_floats, repeat);
    });
}

// ---------------------------------------------------------------------------
// Host-side helpers (scalar arithmetic the reference also does on the host).

double cwlb_capacity_from_s(int32_t s, const cwlb_costs* costs) {
    const cwlb_costs c = costs ? *costs : zero_costs();
    const double edge = c.C_compute_ns + c.C_load_ns;
    const int32_t cs = std::max<int32_t>(1, s);
    if (edge <= 0.0) return std::max(0.0, c.C_atomic_ns);
    return std::max(0.0, c.C_atomic_ns + edge * static_cast<double>(cs));
}

int32_t cwlb_segment_size(const cwlb_costs* costs, double capacity) {
    const cwlb_costs c = costs ? *costs : zero_costs();
    const double wCL = c.C_compute_ns + c.C_load_ns;
    const double q = std::floor((capacity - c.C_atomic_ns) / std::max(1e-30, wCL));
    // double -> int32 as x86-64 converts it: out-of-range and NaN give INT32_MIN.
    const int32_t t = (q >= -2147483648.0 && q < 2147483648.0) ? static_cast<int32_t>(q)
                                                                : std::numeric_limits<int32_t>::min();
    return std::max<int32_t>(1, t);
}

int cwlb_wave_based_s(int64_t nnz, int32_t compute_units, int32_t wave, int32_t* s) {
    return guarded([&] {
        require(s != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null output");
        if (compute_units <= 0 || wave <= 0) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "compute_units and wave must be positive.");
        }
        const uint64_t n = static_cast<uint64_t>(nnz);
        const uint64_t d = static_cast<uint64_t>(compute_units) * static_cast<uint64_t>(wave);
        uint64_t v = (n + d - 1) / d;
        v = std::max<uint64_t>(1, v);
        v = std::min<uint64_t>(v, static_cast<uint64_t>(std::numeric_limits<int32_t>::max()));
        *s = static_cast<int32_t>(v);
    });
}

void cwlb_recommended_candidate_w(uint64_t nnz, int32_t out[3]) {
    // nnz thresholds and the leading candidate of each band; the other two
    // candidates halve it (main.cpp:87-95).
    static const uint64_t limit[] = {100000ULL, 500000ULL, 1000000ULL, 5000000ULL,
                                     10000000ULL, 50000000ULL};
    static const int32_t lead[] = {64, 128, 256, 512, 1024, 4096, 8192};
    int i = 0;
    while (i < 6 && nnz >= limit[i]) ++i;
    out[0] = lead[i];
    out[1] = lead[i] / 2;
    out[2] = lead[i] / 4;
}

int cwlb_save_costs(const cwlb_costs* costs, const char* path, int32_t append,
                    int32_t precision) {
    namespace fs = std::filesystem;
    if (!costs || !path || !*path) {
        g_last_error = "empty cost-file path";
        return CWLB_ERR_RUNTIME;
    }
    std::error_code ec;
    const fs::path p(path);
    if (p.has_parent_path()) {
        const fs::path dir = p.parent_path();
        if (fs::exists(dir, ec) && !fs::is_directory(dir, ec)) {
            g_last_error = "cost-file parent is not a directory";
            return CWLB_ERR_RUNTIME;
        }
        if (!fs::exists(dir, ec) && !fs::create_directories(dir, ec) && ec) {
            g_last_error = "cannot create the cost-file directory";
            return CWLB_ERR_RUNTIME;
        }
    }
    std::ofstream ofs(p, std::ios::out | (append ? std::ios::app : std::ios::trunc));
    if (!ofs.is_open()) {
        g_last_error = "cannot open the cost file";
        return CWLB_ERR_RUNTIME;
    }
    ofs << std::fixed << std::setprecision(precision) << costs->C_compute_ns << "\n"
        << costs->C_load_ns << "\n"
        << costs->C_store_ns << "\n"
        << costs->C_atomic_ns << "\n";
    if (!ofs.good()) {
        g_last_error = "cost-file write failed";
        return CWLB_ERR_RUNTIME;
    }
    return CWLB_OK;
}

int cwlb_read_costs(cwlb_costs* costs, const char* path) {
    if (!costs || !path) {
        g_last_error = "null argument";
        return CWLB_ERR_INVALID_ARGUMENT;
    }
    std::ifstream ifs(path);
    double v[4];
    if (!ifs.is_open() || !(ifs >> v[0]) || !(ifs >> v[1]) || !(ifs >> v[2]) || !(ifs >> v[3])) {
        g_last_error = std::string("cannot read microbenchmark cost file: ") + path;
        return CWLB_ERR_RUNTIME;
    }
    costs->C_compute_ns = v[0];
    costs->C_load_ns = v[1];
    costs->C_store_ns = v[2];
    costs->C_atomic_ns = v[3];
    return CWLB_OK;
}

int cwlb_save_costs_per_k(const cwlb_costs* costs, int64_t n, const char* path) {
    namespace fs = std::filesystem;
    if (!path || !*path || n < 0 || (n > 0 && !costs)) {
        g_last_error = "invalid per-K cost table arguments";
        return CWLB_ERR_RUNTIME;
    }
    for (int64_t i = 0; i < n; ++i) {
        if (costs[i].K <= 0) {
            g_last_error = "per-K cost entries need a positive K";
            return CWLB_ERR_RUNTIME;
        }
    }
    std::error_code ec;
    const fs::path p(path);
    if (p.has_parent_path() && !fs::exists(p.parent_path(), ec) &&
        !fs::create_directories(p.parent_path(), ec) && ec) {
        g_last_error = "cannot create the cost-file directory";
        return CWLB_ERR_RUNTIME;
    }
    std::ofstream ofs(p, std::ios::out | std::ios::trunc);
    if (!ofs.is_open()) {
        g_last_error = "cannot open the per-K cost file";
        return CWLB_ERR_RUNTIME;
    }
    ofs << "# K C_compute_ns C_load_ns C_store_ns C_atomic_ns\n" << std::fixed
        << std::setprecision(6);
    for (int64_t i = 0; i < n; ++i) {
        ofs << costs[i].K << ' ' << costs[i].C_compute_ns << ' ' << costs[i].C_load_ns << ' '
            << costs[i].C_store_ns << ' ' << costs[i].C_atomic_ns << "\n";
    }
    if (!ofs.good()) {
        g_last_error = "per-K cost-file write failed";
        return CWLB_ERR_RUNTIME;
    }
    return CWLB_OK;
}

int cwlb_read_costs_per_k(cwlb_costs* costs, int64_t max_entries, const char* path, int64_t* n) {
    if (!path || !n || max_entries < 0 || (max_entries > 0 && !costs)) {
        g_last_error = "null argument";
        return CWLB_ERR_INVALID_ARGUMENT;
    }
    *n = 0;
    std::ifstream ifs(path);
    if (!ifs.is_open()) {
        g_last_error = std::string("cannot read per-K cost file: ") + path;
        return CWLB_ERR_RUNTIME;
    }
    std::string line;
    int64_t count = 0, lineno = 0;
    while (std::getline(ifs, line)) {
        ++lineno;
        const size_t b = line.find_first_not_of(" \t\r");
        if (b == std::string::npos || line[b] == '#') continue;
        std::istringstream ls(line);
        long long k = 0;
        double v[4];
        std::string rest;
        if (!(ls >> k >> v[0] >> v[1] >> v[2] >> v[3]) || (ls >> rest) || k <= 0 ||
            k > INT32_MAX) {
            g_last_error = std::string("malformed per-K cost file line ") +
                           std::to_string(lineno) + ": " + path;
            return CWLB_ERR_RUNTIME;
        }
        if (count < max_entries) {
            cwlb_costs c{};
            c.K = static_cast<int32_t>(k);
            c.C_compute_ns = v[0];
            c.C_load_ns = v[1];
            c.C_store_ns = v[2];
            c.C_atomic_ns = v[3];
            costs[count] = c;
        }
        ++count;
    }
    *n = count;
    if (count > max_entries && max_entries > 0) {
        g_last_error = "per-K cost table larger than the buffer";
        return CWLB_ERR_BUFFER_TOO_SMALL;
    }
    return CWLB_OK;
}

int64_t cwlb_costs_for_k(const cwlb_costs* costs, int64_t n, int64_t K) {
    if (!costs || n <= 0 || K <= 0) return -1;
    int64_t best = -1;
    double best_d = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        if (costs[i].K <= 0) continue;
        const double d = std::fabs(std::log2(static_cast<double>(costs[i].K)) -
                                   std::log2(static_cast<double>(K)));
        if (best < 0 || d < best_d || (d == best_d && costs[i].K > costs[best].K)) {
            best = i;
            best_d = d;
        }
    }
    return best;
}

}  // extern "C"
