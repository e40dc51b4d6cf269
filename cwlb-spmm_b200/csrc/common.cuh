// Internal helpers shared by the CUDA translation units of libcwlb_spmm.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "cwlb_spmm.h"

namespace cwlb {

// Library-internal failure carrying a cwlb_status; converted to a return code
// (and a thread-local message) at the C boundary.
struct Failure : std::runtime_error {
    int code;
    Failure(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Failure(code, msg); }

inline void check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    if (e == cudaErrorMemoryAllocation) {
        fail(CWLB_ERR_OUT_OF_MEMORY, std::string(what) + ": " + cudaGetErrorString(e));
    }
    fail(CWLB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define CWLB_CUDA(call) ::cwlb::check_cuda((call), #call)
#define CWLB_LAUNCH_CHECK(name) ::cwlb::check_cuda(cudaGetLastError(), name)

// A device buffer that grows on demand and is reused across calls.
struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    void* ensure(size_t need) {
        if (need <= bytes) return ptr;
        release();
        size_t want = need < 256 ? 256 : need;
        CWLB_CUDA(cudaMalloc(&ptr, want));
        bytes = want;
        return ptr;
    }
    template <typename T>
    T* as(size_t count) {
        return static_cast<T*>(ensure(count * sizeof(T)));
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct HostStager;  // pinned bounce slots and copy threads (staging.cu)

}  // namespace cwlb

// The context (opaque in the C API).
struct cwlb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    cudaDeviceProp props{};
    cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
    // Host-buffer calls copy their inputs on copy_stream in chunks and start
    // aggregating each chunk's tasks on `stream` as soon as it has arrived.
    static constexpr int kPipeChunks = 8;
    cudaStream_t copy_stream = nullptr;
    // A plan's groups run on copy_stream beside the ungrouped tasks.
    cudaEvent_t plan_fork = nullptr, plan_join = nullptr;
    cudaEvent_t pipe_ready[kPipeChunks] = {};
    cudaEvent_t pipe_t0[kPipeChunks] = {}, pipe_t1[kPipeChunks] = {};
    uint32_t* d_error_flags = nullptr;  // CWLB_DEVERR_* bits raised by kernels
    // Scratch for the host-buffer entry points (inputs/outputs staged on the
    // device) and for the sort / partition pipelines.
    cwlb::DeviceBuffer in_rowoff, in_col, in_val, in_origin, in_H, in_tasks, out_buf;
    cwlb::DeviceBuffer sort_scratch, part_scratch, part_desc, part_tasks, check_scratch;
    // Fragment partials and their plan (CWLB_DETERMINISTIC).
    cwlb::DeviceBuffer det_scratch;
    // Created by the first large copy of pageable caller memory.
    cwlb::HostStager* stager = nullptr;
};

namespace cwlb {

// launch_spmm_mean flag (internal): the caller has already zeroed `out`.
constexpr uint32_t kFlagOutCleared = 1u << 31;
// Warp kernels (one warp per task, or per run of small tasks), not one CTA
// per task: what task_variant_flag gives a long task list.
constexpr uint32_t kFlagWarpTasks = 1u << 29;
// launch_spmm_mean flag (internal): the split rows of a CWLB_ROWS_COVERED call
// have already been zeroed (by an earlier call with n_slots == 0).
constexpr uint32_t kFlagSplitZeroed = 1u << 30;

// Launchers implemented in the .cu files (all asynchronous on ctx->stream).
// The kernel family for a task list of n_tasks: the one `flags` forces
// (CWLB_TASK_PER_WARP, CWLB_TASK_PER_CTA), else CWLB_TASK_PER_CTA for at most
// 128 tasks per SM and kFlagWarpTasks otherwise.  Callers that launch one list
// in pieces (chunks, a launch order over part of it) pass the whole list's
// choice to every piece, so that every row a task covers whole comes out as
// one launch would give it.
uint32_t task_variant_flag(const cwlb_ctx* ctx, int64_t n_tasks, uint32_t flags);
// Tasks per warp run (spmm_run_kernel) for a list of n_tasks over nnz
// nonzeros: 1 (no runs) unless tasks average fewer than 128 nonzeros.
int32_t task_run_length(int64_t nnz, int64_t n_tasks);
void launch_spmm_mean(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                      const int32_t* col, const float* val, const int32_t* origin,
                      const float* H, int64_t h_rows, int64_t K, const cwlb_task* tasks,
                      int64_t n_tasks, float* out, uint32_t flags,
                      const int32_t* sched = nullptr, int64_t n_slots = 0, int32_t run = -1);
// Copies of caller memory for the host-buffer entry points (staging.cu).
// copy_to_device is asynchronous on `s`; once it returns, the source may be
// reused; copy_to_host returns when `dst` holds the data.  Large pageable
// copies go through the context's pinned slots.
void copy_to_device(cwlb_ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t s);
void copy_to_host(cwlb_ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t s);
void destroy_stager(cwlb_ctx* ctx);
// Aggregation plans (plan.cu).
cwlb_plan* plan_create(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                       const int32_t* col, const float* val, const cwlb_task* tasks,
                       int64_t n_tasks, int32_t group_size);
void plan_aggregate(cwlb_plan* p, const int32_t* origin, const float* H, int64_t h_rows, int64_t K,
                    float* out, uint32_t flags);
void plan_destroy(cwlb_plan* p);
// True when every one of the `count` device floats is exactly 1.0f
// (synchronous; d_flag is one word of device scratch) (spmm.cu).  Kernels
// given NULL values treat every value as 1.0f.
bool values_all_one(cwlb_ctx* ctx, const float* d_val, size_t count, unsigned int* d_flag);
// Float64 reference of the aggregation over an unsorted CSR (spmm.cu).
void launch_spmm_mean_reference(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                                const int32_t* col, const float* val, const float* H,
                                int64_t h_rows, int64_t K, float* out);
void run_tasks_check(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                     const cwlb_task* tasks, int64_t n_tasks, int64_t* bad_tasks,
                     int64_t* uncovered_rows, int64_t* nnz_errors);
void launch_sort_by_degree(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                           const int32_t* col, const float* val, int32_t* origin,
                           int32_t* new_rowoff, int32_t* new_col, float* new_val);
// Stable LSD radix sort of (key, value) pairs by the low `bits` bits of the
// keys, 8 bits per pass, in place on ctx's stream (reorder.cu); scratch holds
// radix_sort_pairs_scratch_bytes(n, SM count) bytes.
size_t radix_sort_pairs_scratch_bytes(int32_t n, int sm_count);
void radix_sort_pairs(cwlb_ctx* ctx, uint32_t* keys, int32_t* vals, int32_t n, int bits,
                      void* scratch);
// Returns the number of tasks; the tasks are in ctx->part_tasks.
int64_t run_partition(cwlb_ctx* ctx, int32_t n_rows, const int32_t* d_rowoff,
                      const cwlb_costs& costs, double capacity);
// The four calibration microbenchmarks (calibrate.cu).
void measure_costs(cwlb_ctx* ctx, int K, int repeat, int WI, int data_MB, int writers,
                   cwlb_costs* out);
// Random-row gather rate over a buffer_MB MiB device buffer, GB/s (calibrate.cu).
double measure_gather_gbs(cwlb_ctx* ctx, int buffer_MB, int row_floats, int repeat);
// Sets the calling thread's cwlb_last_error() message (defined in capi.cu).
void set_last_error(const std::string& msg);

}  // namespace cwlb
