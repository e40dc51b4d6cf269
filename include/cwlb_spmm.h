/*
 * cwlb_spmm.h - C ABI of the B200 (sm_100a) CWLB-SpMM library.
 *
 * The hot path is FP32 CSR mean aggregation
 *     out[origin[r], k] = (1 / deg_r) * sum_{j in row r} value_j * H[col_j, k]
 * over a degree-reordered CSR, driven by cost-weighted task descriptors.
 * Every entry point below replaces one interface of the reference
 * (hhx-C/CWLB-SpMM); the comment on each names the reference code by
 * file:line, relative to that project's root.  The C++17 drop-in API in
 * cwlb-spmm_b200/host/include/ (Matrix.h, utils.h, parallelMatrix.h, ...)
 * is a thin layer over these functions.
 *
 * Conventions
 *   - Every function returns a cwlb_status; on failure cwlb_last_error()
 *     returns the message of the calling thread's last failure.  Status codes
 *     map one-to-one onto the C++ exception types the reference throws.
 *   - "host" pointers are ordinary (pageable or pinned) host memory;
 *     "d_" pointers are device memory of the context's device.
 *   - *_device entry points are asynchronous on the context's stream; all
 *     others are synchronous (they return when results are in host memory),
 *     as the reference's q.wait() based functions are.
 *   - A context is bound to one device and is not thread-safe; use one
 *     context per GPU and per host thread.
 *   - The library owns only its scratch memory; it never frees caller memory.
 *   - No entry point falls back to a CPU implementation.  Without a usable
 *     CUDA device cwlb_ctx_create fails with CWLB_ERR_NO_DEVICE.
 */
#ifndef CWLB_SPMM_H_
#define CWLB_SPMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum cwlb_status {
    CWLB_OK = 0,
    CWLB_ERR_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
    CWLB_ERR_RUNTIME = 2,          /* reference: std::runtime_error */
    CWLB_ERR_OVERFLOW = 3,         /* reference: std::overflow_error */
    CWLB_ERR_CUDA = 4,             /* a CUDA runtime call failed */
    CWLB_ERR_NO_DEVICE = 5,        /* no usable CUDA device */
    CWLB_ERR_BUFFER_TOO_SMALL = 6, /* output capacity too small; size reported */
    CWLB_ERR_OUT_OF_MEMORY = 7     /* device allocation failed */
} cwlb_status;

/* ParallelDataWeighted (include/utils.h:15-20): one task = a half-open range
 * of reordered rows plus the nnz offsets that bound its first and last row. */
typedef struct cwlb_task {
    int32_t row_start;        /* first reordered row, inclusive */
    int32_t row_end;          /* last reordered row, exclusive */
    int32_t first_row_offset; /* nnz offset within the first row */
    int32_t last_row_nnz;     /* end offset within the last row; 0 = full degree */
} cwlb_task;

/* SpmmCostParams (include/utils.h:23-33): calibrated weights (ns x 10 per
 * operation) plus the calibration metadata. */
typedef struct cwlb_costs {
    double C_compute_ns;
    double C_load_ns;
    double C_store_ns;
    double C_atomic_ns;
    int32_t K;
    int32_t WI;
    int32_t repeat;
    int32_t atomic_writers_per_addr;
} cwlb_costs;

typedef struct cwlb_ctx cwlb_ctx;

/* Message of the calling thread's last failing call ("" if none). */
const char* cwlb_last_error(void);
/* Library version string. */
const char* cwlb_version(void);

/* ---------------------------------------------------------------- context */

/* Replaces sycl::queue(gpu_selector_v, enable_profiling) (main.cpp:514-516,
 * weightCost.cpp:44-46): binds CUDA device `device` and creates a stream. */
int cwlb_ctx_create(int device, cwlb_ctx** ctx);
int cwlb_ctx_destroy(cwlb_ctx* ctx);
/* Use an existing cudaStream_t (passed as void*) instead of the own stream. */
int cwlb_ctx_set_stream(cwlb_ctx* ctx, void* cuda_stream);
void* cwlb_ctx_stream(cwlb_ctx* ctx);
/* Replaces q.wait(). */
int cwlb_ctx_synchronize(cwlb_ctx* ctx);
/* Device-side error flags raised by kernels since the last call (bit mask of
 * CWLB_DEVERR_*); reading clears them.  Kernels never fault on bad indices:
 * they skip the offending entry and raise a flag instead. */
int cwlb_ctx_take_device_errors(cwlb_ctx* ctx, uint32_t* flags);
#define CWLB_DEVERR_COL_RANGE 1u    /* a column index outside [0, h_rows) */
#define CWLB_DEVERR_ROW_RANGE 2u    /* a task row outside [0, n_rows) */
#define CWLB_DEVERR_OFFSETS 4u      /* row offsets not monotone or beyond nnz */
#define CWLB_DEVERR_ORIGIN_RANGE 8u /* an origin id outside [0, n_rows) */
/* Device queries the reference reads from sycl::device::get_info:
 * max_work_group_size (parallelMatrix.cpp:76-77, main.cpp:359-361; 1024 on
 * CUDA), max_compute_units (main.cpp:535-536, 718-719; the SM count),
 * local_mem_size (parallelMatrix.cpp:349-350) and the device name. */
int cwlb_device_info(cwlb_ctx* ctx, int64_t* max_work_group_size, int32_t* compute_units,
                     int64_t* local_mem_size, char* name, size_t name_capacity);

/* ------------------------------------------------------------------- SpMM */

/* spmmKernel (include/parallelMatrix.h:13-20, src/parallelMatrix.cpp:63-254).
 * Host buffers.  Inputs: the reordered CSR (row_offset[n_rows+1], col_ind and
 * value[nnz], origin_local[n_rows]), H (h_rows x K, row-major) and the task
 * list.  Writes out (n_rows x K, row-major, ORIGINAL row order; rows no task
 * covers are zero) and *time_us (device time of the aggregation kernels, in
 * microseconds, excluding transfers as the reference's event time does).
 * dim_hint is unused and local_dimension is accepted for signature parity
 * (the reference uses it only to size its local-memory staging tile).
 * Errors: K > 1024 -> CWLB_ERR_INVALID_ARGUMENT (use the large-K entry);
 * K == 0 or no tasks -> zero output and *time_us = 0, as the reference. */
int cwlb_spmm_kernel(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                     const int32_t* col_ind, const float* value, const int32_t* origin_local,
                     const float* H, int64_t h_rows, int64_t K, int32_t dim_hint,
                     int32_t local_dimension, const cwlb_task* tasks, int64_t n_tasks,
                     float* out, double* time_us);

/* spmmKernelLargeKFallback (include/parallelMatrix.h:25-32,
 * src/parallelMatrix.cpp:264-683): same contract; requires K > 1024
 * (otherwise CWLB_ERR_INVALID_ARGUMENT, as the reference). */
int cwlb_spmm_kernel_large_k(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                             const int32_t* row_offset, const int32_t* col_ind,
                             const float* value, const int32_t* origin_local, const float* H,
                             int64_t h_rows, int64_t K, int32_t dim_hint,
                             int32_t local_dimension, const cwlb_task* tasks, int64_t n_tasks,
                             float* out, double* time_us);

/* Device-resident form of both entry points (any K >= 0), asynchronous on the
 * context's stream, so that the CSR, H and tasks stay resident across
 * launches (the reference's 70-launch timing loop, main.cpp:372-406).
 * flags: 0 -> out is zero-filled first (reference semantics);
 * CWLB_ROWS_COVERED -> the caller asserts that the tasks cover every row
 * (see cwlb_tasks_check); the kernels then write every output row themselves
 * and the full zero-fill is skipped.
 * d_value may be NULL: every value is then 1.0 (the reference's text loader
 * gives every stored entry the value 1, src/data.cpp:115) and the kernels
 * need not read values; the result equals passing an array of ones (bit for
 * bit where the merge order is fixed).  On invalid input the two differ: an
 * out-of-range column raises CWLB_DEVERR_COL_RANGE either way, but with NULL
 * values its row is not skipped (the output is then undefined).
 * CWLB_DETERMINISTIC -> rows split across tasks are merged in a fixed order
 * (fragment partials kept in context scratch of up to 2 x n_tasks x K floats,
 * then summed per row in task order, in blocks of 64 fragments) instead of
 * with float atomics, so repeated calls give bit-identical outputs; the
 * reference's atomics (src/parallelMatrix.cpp:219-234) promise no order. */
#define CWLB_ROWS_COVERED 1u
#define CWLB_DETERMINISTIC 2u
/* Kernel variant (K a multiple of 4, H and out 16-byte aligned): one warp per
 * task; when the list holds at most 128 tasks per SM (a large S, a small
 * graph), one 8-warp CTA per task, a hub fragment then split over the CTA and
 * reduced through shared memory; when tasks average fewer than 128 nonzeros
 * (a small S), one warp per run of consecutive tasks, consecutive fragments
 * of one row summed in registers and written once (fewer float atomics, less
 * rounding).  A row that one lane group sums alone is summed in nonzero order
 * in every variant, so those rows are bit-identical between them.  These
 * flags force one warp per task (no runs) or one CTA per task (tuning,
 * tests); not both. */
#define CWLB_TASK_PER_WARP 4u
#define CWLB_TASK_PER_CTA 8u
int cwlb_spmm_mean_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                          const int32_t* d_row_offset, const int32_t* d_col_ind,
                          const float* d_value, const int32_t* d_origin_local, const float* d_H,
                          int64_t h_rows, int64_t K, const cwlb_task* d_tasks, int64_t n_tasks,
                          float* d_out, uint32_t flags);

/* Aggregation plan: a task list prepared once for many launches (the
 * reference's 70-launch timing loop, main.cpp:372-406, or one graph layer
 * after another); no counterpart in the reference.  Same results as
 * cwlb_spmm_mean_device on the same inputs: every task covers exactly its
 * own nonzeros and is written as the task kernel writes it; only the order
 * of additions inside a row fragment may differ (within the same tolerance),
 * and rows that one task covers whole are computed by the task kernel.
 * Building (synchronous) groups single-row fragment tasks of neighbouring
 * rows, `group_size` per group (0: the library's choice, 4; 2-4: 4; 5-8: 8;
 * 1: no groups), and stores each group's merged union of nonzeros in runs of
 * equal member mask; one warp then aggregates a group, loading each distinct
 * H row once, summing a run in registers and adding the sum to the run's
 * members.  Groups are kept only when every grouped value is 1.0f, every
 * grouped fragment's columns are non-decreasing and the union saves enough
 * loads; otherwise (and, per call, for K not in {32, 64, 128}, unaligned H or
 * out, or CWLB_DETERMINISTIC) the plan runs the task kernel over all tasks,
 * and cwlb_plan_info's *off_reason says why (CWLB_PLAN_* bits).  The plan
 * keeps the CSR and task pointers: they must stay valid and unchanged until
 * cwlb_plan_destroy.  Its own buffers are device memory it allocates. */
#define CWLB_PLAN_DISABLED 1u       /* group_size 1 */
#define CWLB_PLAN_FEW_FRAGMENTS 2u  /* too few single-row fragment tasks */
#define CWLB_PLAN_VALUES 4u         /* a grouped value is not 1.0f */
#define CWLB_PLAN_UNSORTED 8u       /* a grouped fragment's columns decrease */
#define CWLB_PLAN_NO_REUSE 16u      /* the union would save too few loads */
typedef struct cwlb_plan cwlb_plan;
int cwlb_plan_create(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* d_row_offset,
                     const int32_t* d_col_ind, const float* d_value, const cwlb_task* d_tasks,
                     int64_t n_tasks, int32_t group_size, cwlb_plan** out);
/* Tasks in groups, their nonzeros, the union entries that replace them, the
 * group size in use (0: none) and the CWLB_PLAN_* reasons groups are off. */
int cwlb_plan_info(const cwlb_plan* plan, int64_t* grouped_tasks, int64_t* grouped_nnz,
                   int64_t* union_entries, int32_t* group_size, uint32_t* off_reason);
/* One aggregation with cwlb_spmm_mean_device's contract (out zero-filled
 * first, or CWLB_ROWS_COVERED / CWLB_DETERMINISTIC as there), asynchronous
 * on the plan's context stream. */
int cwlb_plan_aggregate_device(cwlb_plan* plan, const int32_t* d_origin_local, const float* d_H,
                               int64_t h_rows, int64_t K, float* d_out, uint32_t flags);
int cwlb_plan_destroy(cwlb_plan* plan);

/* Validates a device task list against a reordered CSR (no counterpart in the
 * reference, which trusts its partitioner): *bad_tasks counts tasks whose rows
 * fall outside [0, n_rows); *uncovered_rows counts rows in no task's row
 * range; *nnz_coverage_errors counts nonzeros not covered exactly once.
 * Synchronous. */
int cwlb_tasks_check(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* d_row_offset,
                     const cwlb_task* d_tasks, int64_t n_tasks, int64_t* bad_tasks,
                     int64_t* uncovered_rows, int64_t* nnz_coverage_errors);

/* ---------------------------------------------------------- degree reorder */

/* sortCSRByDegreeDPLCPU (main.cpp:197-278) on the GPU: rows ordered by
 * (degree ascending, original id ascending), new offsets = inclusive scan of
 * the sorted degrees, rows copied unchanged.  Bit-identical to the reference.
 * Host buffers: origin_local[n_rows], sorted_row_offset[n_rows+1],
 * sorted_col_ind[nnz], sorted_value[nnz].  n_rows == 0 returns an empty
 * result.  Errors: CWLB_ERR_RUNTIME when row_offset[n_rows] != nnz. */
int cwlb_sort_by_degree(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                        const int32_t* col_ind, const float* value, int32_t* origin_local,
                        int32_t* sorted_row_offset, int32_t* sorted_col_ind,
                        float* sorted_value);
/* Device-buffer form (asynchronous). */
int cwlb_sort_by_degree_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                               const int32_t* d_row_offset, const int32_t* d_col_ind,
                               const float* d_value, int32_t* d_origin_local,
                               int32_t* d_sorted_row_offset, int32_t* d_sorted_col_ind,
                               float* d_sorted_value);

/* ------------------------------------------------------------- partitioner */

/* costWeightedTaskPartitioning (include/utils.h:57-60,
 * src/utils.cpp:832-1021) on the GPU, bit-identical task list.
 * row_offset: the reordered CSR's offsets (host, n_rows+1).  tasks may be
 * NULL to query the count; if max_tasks is smaller than the count the call
 * returns CWLB_ERR_BUFFER_TOO_SMALL with *n_tasks set. */
int cwlb_partition(cwlb_ctx* ctx, int32_t n_rows, const int32_t* row_offset,
                   const cwlb_costs* costs, double capacity, cwlb_task* tasks,
                   int64_t max_tasks, int64_t* n_tasks);
/* Device form: reads d_row_offset, writes the task list into context-owned
 * device memory returned in *d_tasks (valid until the next partition call on
 * this context) and its length in *n_tasks.  Synchronises once to learn the
 * task count. */
int cwlb_partition_device(cwlb_ctx* ctx, int32_t n_rows, const int32_t* d_row_offset,
                          const cwlb_costs* costs, double capacity, cwlb_task** d_tasks,
                          int64_t* n_tasks);

/* Device partitioner that allocates nothing.  It has no counterpart in the
 * reference.  It is for callers that cannot let a library call cudaMalloc or
 * cudaFree: their device memory is owned by another allocator (a framework's
 * caching allocator, or a pool a server sizes once at start-up to keep its
 * footprint fixed), and those calls would also synchronise the device in the
 * middle of their pipelines.  Such callers pass the input offsets and the
 * output task buffer; the scratch lives in one fixed 8 MiB device array that
 * every GPU loading this library holds until the process exits.
 * Same result as cwlb_partition_device (bit-identical task list), written to
 * d_tasks (capacity max_tasks; CWLB_ERR_BUFFER_TOO_SMALL with *n_tasks set
 * when it does not fit).  Limits: n_rows <= CWLB_NOALLOC_MAX_ROWS and at most
 * CWLB_NOALLOC_MAX_RUNS distinct row degrees; larger inputs are rejected with
 * CWLB_ERR_INVALID_ARGUMENT.  Runs on `cuda_stream` (a cudaStream_t; NULL is
 * the default stream) of the calling thread's current device, needs no
 * context, and synchronises that stream twice to learn sizes.  The first call
 * on each device looks up the scratch array's device address; make that first
 * call before any stream capture that includes this function.  All calls share
 * the one array: calls whose work overlaps on the GPU race and must be
 * serialised by the caller. */
#define CWLB_NOALLOC_MAX_ROWS 1048576
#define CWLB_NOALLOC_MAX_RUNS 16384
int cwlb_partition_device_noalloc(void* cuda_stream, int32_t n_rows, const int32_t* d_row_offset,
                                  const cwlb_costs* costs, double capacity, cwlb_task* d_tasks,
                                  int64_t max_tasks, int64_t* n_tasks);

/* -------------------------------------------------------------- multi-GPU */

/* The reference runs its whole pipeline on one sycl::queue (main.cpp:514-516):
 * sortCSRByDegreeDPLCPU (main.cpp:197-278), costWeightedTaskPartitioning
 * (src/utils.cpp:832-1021) and spmmKernel (src/parallelMatrix.cpp:63-254).
 * The functions below run that pipeline on several GPUs of one node without
 * a data exchange: shard s takes a contiguous block of ORIGINAL rows, sorts
 * and partitions it on its own GPU (the reference's algorithms applied to
 * the block, so a shard's task list is the partition of its block, not a
 * slice of the whole graph's), and aggregates it with H replicated; its
 * output is the block's rows of the original-order result. */

/* Cost-balanced contiguous row shards: bounds[0] = 0, bounds[n_shards] =
 * n_rows, shard s = original rows [bounds[s], bounds[s+1]).  The cut after
 * shard s-1 follows the first row whose inclusive prefix sum of the
 * whole-row weight (Cc + Cl) * deg + Cs (src/utils.cpp:850-852; sequential
 * float64) reaches total * s / n_shards.  Host code; no device needed. */
int cwlb_shard_bounds(int32_t n_rows, const int32_t* row_offset, const cwlb_costs* costs,
                      int32_t n_shards, int32_t* bounds);

/* The same rule re-weighted by measured shard times: every row of shard g
 * under `bounds` (n_shards + 1 cut points, from 0 to n_rows, non-decreasing)
 * weighs its whole-row weight times shard_time[g] / W_g, W_g being the shard's
 * summed weight under that cut (shards without weight keep factor 1), and
 * new_bounds receives the cut of the re-weighted prefix sum (same sequential
 * float64 rule; new_bounds may alias bounds).  The kernel's real cost per row
 * differs from the modelled one by degree class (on a B200, a row of a few
 * nonzeros costs about as much as 17 nonzeros of a hub row at K = 64); the
 * times of one aggregation of each shard fold that back into the cut.  Every
 * GPU of a job must pass the same times (e.g. all-gathered) to get the same
 * cut.  CWLB_ERR_INVALID_ARGUMENT for bad bounds, or a non-positive or
 * non-finite time of a shard with weight.  Host code; no device needed. */
int cwlb_shard_bounds_rebalance(int32_t n_rows, const int32_t* row_offset,
                                const cwlb_costs* costs, int32_t n_shards,
                                const int32_t* bounds, const double* shard_time,
                                int32_t* new_bounds);

typedef struct cwlb_shard cwlb_shard;

/* Builds shard `shard` of `n_shards` on ctx's device from the caller's whole
 * UNSORTED CSR (host buffers, original row order): cuts the shards as
 * cwlb_shard_bounds, copies the block's rows to the device, sorts them by
 * degree, partitions them at `capacity` and checks the task list once; the
 * result stays resident until cwlb_shard_destroy.  Synchronous.
 * Errors: CWLB_ERR_RUNTIME when row_offset[n_rows] != nnz (the reference's
 * message), CWLB_ERR_INVALID_ARGUMENT for bad offsets or shard indices. */
int cwlb_shard_create(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                      const int32_t* col_ind, const float* value, const cwlb_costs* costs,
                      double capacity, int32_t shard, int32_t n_shards, cwlb_shard** out);
/* cwlb_shard_create with the cut given: `cut` holds n_shards + 1 host ints
 * from 0 to n_rows, non-decreasing (e.g. from cwlb_shard_bounds_rebalance);
 * NULL cuts as cwlb_shard_bounds. */
int cwlb_shard_create_cut(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                          const int32_t* col_ind, const float* value, const cwlb_costs* costs,
                          double capacity, const int32_t* cut, int32_t shard, int32_t n_shards,
                          cwlb_shard** out);
/* Same, with the whole CSR already in ctx's device memory (one process per
 * GPU, each holding the graph); the block is sorted straight from it. */
int cwlb_shard_create_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                             const int32_t* d_row_offset, const int32_t* d_col_ind,
                             const float* d_value, const cwlb_costs* costs, double capacity,
                             int32_t shard, int32_t n_shards, cwlb_shard** out);
/* cwlb_shard_create_device with the cut given, as cwlb_shard_create_cut. */
int cwlb_shard_create_device_cut(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                                 const int32_t* d_row_offset, const int32_t* d_col_ind,
                                 const float* d_value, const cwlb_costs* costs, double capacity,
                                 const int32_t* cut, int32_t shard, int32_t n_shards,
                                 cwlb_shard** out);
/* The shard's original rows [*row_begin, *row_end), its nonzeros, task count
 * and the segment size S the partitioner derived; NULL outputs are skipped. */
int cwlb_shard_info(const cwlb_shard* shard, int32_t* row_begin, int32_t* row_end, int32_t* nnz,
                    int64_t* n_tasks, int32_t* segment_size);
/* Device pointer to the shard's task list (n_tasks entries, indices into the
 * shard's own degree-sorted rows). */
int cwlb_shard_tasks(const cwlb_shard* shard, const cwlb_task** d_tasks);
/* d_out[(r - row_begin) * K + k] = mean aggregation of original row r, for
 * the shard's rows, with d_H (h_rows x K, row-major, all rows of H) on ctx's
 * device.  flags: 0 or CWLB_DETERMINISTIC.  Asynchronous on ctx's stream. */
int cwlb_shard_aggregate_device(cwlb_shard* shard, const float* d_H, int64_t h_rows, int64_t K,
                                float* d_out, uint32_t flags);
int cwlb_shard_destroy(cwlb_shard* shard);

/* The whole pipeline over n_gpus contexts (one per GPU, each used by one
 * host thread that this call starts): from the caller's UNSORTED host CSR
 * and host H to the host output `out` (n_rows x K, ORIGINAL row order), as
 * the reference's main.cpp:530-531 + 352-391 computes it on one device.
 * *time_us receives the largest per-GPU device time of the aggregation
 * kernels (transfers, sort and partition excluded, as the reference's
 * kernel time).  Synchronous. */
int cwlb_spmm_mean_multi(cwlb_ctx* const* ctxs, int32_t n_gpus, int32_t n_rows, int32_t nnz,
                         const int32_t* row_offset, const int32_t* col_ind, const float* value,
                         const float* H, int64_t h_rows, int64_t K, const cwlb_costs* costs,
                         double capacity, float* out, double* time_us);

/* All-gather of a row-sharded matrix across the contexts' GPUs: d_X[g] is a
 * rows x K row-major buffer on ctxs[g]'s device holding valid rows
 * [bounds[g], bounds[g+1]) (e.g. the rows that GPU aggregated in a previous
 * layer); afterwards every buffer holds all rows.  One peer copy per
 * (source, destination) pair over NVLink, ordered on the contexts' streams:
 * it starts after the work already queued on every stream, and later work
 * on any of the streams starts after every copy.  Asynchronous. */
int cwlb_gather_rows_multi(cwlb_ctx* const* ctxs, int32_t n_gpus, float* const* d_X,
                           int64_t rows, int64_t K, const int32_t* bounds);

/* ----------------------------------------------------- S-selection helpers */

/* capacity_from_s (main.cpp:281-292). */
double cwlb_capacity_from_s(int32_t s, const cwlb_costs* costs);
/* The segment size S the partitioner derives from a capacity
 * (src/utils.cpp:859-864). */
int32_t cwlb_segment_size(const cwlb_costs* costs, double capacity);
/* wave_based_s (main.cpp:295-321); CWLB_ERR_INVALID_ARGUMENT for
 * compute_units <= 0 or wave <= 0. */
int cwlb_wave_based_s(int64_t nnz, int32_t compute_units, int32_t wave, int32_t* s);
/* recommended_candidate_w (main.cpp:87-95). */
void cwlb_recommended_candidate_w(uint64_t nnz, int32_t out[3]);

/* ------------------------------------------------------------ calibration */

/* measure_spmm_costs (include/utils.h:47-54, src/utils.cpp:342-829), the
 * costWrite calibration, as CUDA microbenchmarks on this context's device:
 * compute (K dependent FMAs per thread), load (32-lane groups reading random
 * K-float rows of a data_MB_for_load MiB array), store (K floats per thread),
 * atomic (128-thread groups, atomic_target_writers groups per row, float atomic
 * adds).  Each runs 20 untimed and `repeat` timed launches; results are
 * nanoseconds per operation times 10, as in the reference.  The reference's
 * defaults are K=128, repeat=500, WI=131072, data_MB_for_load=512, writers=8.
 * CWLB_ERR_INVALID_ARGUMENT if any parameter is not positive. */
int cwlb_measure_spmm_costs(cwlb_ctx* ctx, int32_t K, int32_t repeat, int32_t WI,
                            int32_t data_MB_for_load, int32_t atomic_target_writers,
                            cwlb_costs* out);

/* Gather-rate microbenchmark (no reference counterpart; it supplies the
 * ceiling for the aggregation's roofline).  Groups of lanes read whole rows of
 * row_floats floats (the rows of X at K = row_floats), chosen uniformly at
 * random among the largest power-of-two number of rows that fits in buffer_MB
 * MiB of device memory, through the read-only data path, with eight 16-byte
 * loads in flight per thread as in the aggregation; as many CTAs of 256
 * threads as fit on every SM, about 4 GB per launch, 20 untimed and `repeat`
 * timed launches.  *gbs
 * receives bytes gathered / mean launch time in GB/s.  A buffer that fits in
 * the 126 MB L2 (e.g. 48 MiB) gives the rate for rows served from L2; one far
 * larger gives the rate for rows served from HBM.
 * CWLB_ERR_INVALID_ARGUMENT unless buffer_MB and repeat are positive, the
 * buffer holds two rows and row_floats is 4 times a power of two, at most 1024. */
int cwlb_measure_gather_gbs(cwlb_ctx* ctx, int32_t buffer_MB, int32_t row_floats,
                            int32_t repeat, double* gbs);

/* ------------------------------------------------------------- validation */

/* Float64 reference of the mean aggregation over an UNSORTED CSR (the
 * caller's original row order): d_out[r, k] = (float)((1/deg_r) *
 * sum_j value_j * H[col_j, k]) with the row's nonzeros summed in order in
 * double, one warp per row; empty rows give 0.  It shares nothing with the
 * sort, the partitioner or the task kernels, so it checks the whole path.
 * No counterpart in the reference, whose validate_custom_csr_result compares
 * against a result the caller supplies (src/utils.cpp:1117-1265); the
 * cwlb-spmm CLI's --verify uses this to produce that result on the device.
 * Asynchronous on the context's stream; bad indices raise device error flags
 * as the aggregation kernels do. */
int cwlb_spmm_mean_reference_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                                    const int32_t* d_row_offset, const int32_t* d_col_ind,
                                    const float* d_value, const float* d_H, int64_t h_rows,
                                    int64_t K, float* d_out);

/* validate_custom_csr_result (src/utils.cpp:1117-1265) on host arrays:
 * compares `result` with `reference` element by element (NaN matches only
 * NaN, an infinity only the same infinity, finite values within
 * abs_tolerance) and prints, like the reference, a pass line or up to 10
 * mismatches with the CSR row (row_offset has row_offset_len entries) and the
 * first 5 entries of the dense matrix's column; shape problems and a bad
 * tolerance are reported on stderr.  *passed receives 1 or 0.  Host code: no
 * context or device is needed. */
int cwlb_validate_result(const float* result, int64_t result_rows, int64_t result_cols,
                         const float* reference, int64_t reference_rows, int64_t reference_cols,
                         const int32_t* row_offset, int64_t row_offset_len,
                         const int32_t* col_ind, const float* value, const float* dense,
                         int64_t dense_rows, int64_t dense_cols, float abs_tolerance,
                         int32_t* passed);

/* ------------------------------------------------------------- cost files */

/* save_costs_one_per_line (src/utils.cpp:1024-1075): four lines, fixed
 * notation with `precision` digits, order compute, load, store, atomic;
 * creates the parent directory.  Returns CWLB_ERR_RUNTIME on failure. */
int cwlb_save_costs(const cwlb_costs* costs, const char* path, int32_t append,
                    int32_t precision);
/* read_costs_one_per_line (src/utils.cpp:1077-1092). */
int cwlb_read_costs(cwlb_costs* costs, const char* path);

/* Per-K cost table: an extension of the cost file (the reference calibrates at
 * one K, 128 by default) with one line "K C_compute C_load C_store C_atomic"
 * per calibrated row width, costs in fixed notation with 6 digits; lines that
 * start with '#' are comments.  cwlb_save_costs_per_k writes the n entries in
 * the given order (their K fields must be positive), creating the parent
 * directory.  cwlb_read_costs_per_k sets *n to the number of entries in the
 * file and copies up to max_entries of them into `costs` (NULL with
 * max_entries 0 only counts); only K and the four costs are filled.  Both
 * return CWLB_ERR_RUNTIME on I/O or format errors; reading returns
 * CWLB_ERR_BUFFER_TOO_SMALL when the file holds more than max_entries. */
int cwlb_save_costs_per_k(const cwlb_costs* costs, int64_t n, const char* path);
int cwlb_read_costs_per_k(cwlb_costs* costs, int64_t max_entries, const char* path, int64_t* n);
/* Index of the entry whose K is nearest to K on a log2 scale (ties go to the
 * larger K); -1 for an empty table or K <= 0. */
int64_t cwlb_costs_for_k(const cwlb_costs* costs, int64_t n, int64_t K);

#ifdef __cplusplus
}
#endif

#endif /* CWLB_SPMM_H_ */
