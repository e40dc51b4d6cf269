// Mean aggregation over several GPUs of one node.
//
// The reference runs on one sycl::queue (main.cpp:514-516); this file spreads
// its whole per-graph pipeline (sortCSRByDegreeDPLCPU, main.cpp:197-278 ->
// costWeightedTaskPartitioning, src/utils.cpp:832-1021 -> spmmKernel,
// src/parallelMatrix.cpp:63-254) over G GPUs without a data exchange:
//
//   * shard s owns a contiguous block of ORIGINAL rows [b_s, b_{s+1}), cut
//     where the prefix sum of the whole-row weight (Cc + Cl) * deg + Cs (the
//     weight the reference's partitioner gives a row, src/utils.cpp:850-852)
//     crosses s/G of the total, so the shards carry equal partitioner cost;
//   * each GPU sorts its block by degree, partitions it with the reference's
//     greedy and aggregates it with the dense input H replicated; its output
//     is rows [b_s, b_{s+1}) of the original-order result, so the slices are
//     disjoint and need no permutation or reduction afterwards;
//   * when H arrives row-sharded (each GPU holding the rows it produced in a
//     previous layer), cwlb_gather_rows_multi rebuilds it on every GPU with
//     peer copies over NVLink before the aggregation.
//
// A shard's task list is the reference's partition of ITS block; it differs
// from a partition of the whole graph (tasks never straddle a shard cut).
#include <algorithm>
#include <cmath>
#include <exception>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

struct cwlb_shard {
    cwlb_ctx* ctx = nullptr;
    int32_t shard = 0, n_shards = 1;
    int32_t row_begin = 0, row_end = 0;  // original rows of the shard
    int32_t n = 0, nnz = 0;
    int32_t segment = 0;                 // S the partitioner derived
    int64_t n_tasks = 0;
    uint32_t flags = 0;                  // CWLB_ROWS_COVERED once checked
    bool unit = false;                   // every value is 1.0: kernels read none
    cwlb::DeviceBuffer origin, rowoff, col, val, tasks;
};

namespace cwlb {
namespace {

template <typename F>
int guarded_multi(F&& f) {
    try {
        f();
        return CWLB_OK;
    } catch (const Failure& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return CWLB_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return CWLB_ERR_RUNTIME;
    }
}

void need(bool ok, int code, const std::string& msg) {
    if (!ok) fail(code, msg);
}

// Cut points of the cost-balanced row shards.  The arithmetic is sequential
// float64, multiply and add rounded separately (this file's host code is
// built with -ffp-contract=off), so the cuts are reproducible bit for bit.
// With old_bounds / scale, the weight of every row of old shard g is
// multiplied by scale[g] (the rebalancing cut).
void shard_bounds_host(int32_t n_rows, const int32_t* rowoff, double edge_w, double store_w,
                       int32_t n_shards, int32_t* bounds, const int32_t* old_bounds = nullptr,
                       const double* scale = nullptr) {
    std::vector<double> cum(static_cast<size_t>(n_rows));
    double acc = 0.0;
    int32_t g = 0;
    for (int32_t r = 0; r < n_rows; ++r) {
        const double deg = static_cast<double>(static_cast<int64_t>(rowoff[r + 1]) - rowoff[r]);
        double w = deg * edge_w + store_w;
        if (scale) {
            while (r >= old_bounds[g + 1]) ++g;
            w = w * scale[g];
        }
        acc = acc + w;
        cum[static_cast<size_t>(r)] = acc;
    }
    const double total = n_rows > 0 ? cum.back() : 0.0;
    bounds[0] = 0;
    for (int32_t k = 1; k < n_shards; ++k) {
        const double target = total * static_cast<double>(k) / static_cast<double>(n_shards);
        // First row whose inclusive prefix reaches the target; the cut
        // follows it, so the row that crosses k/G stays in the earlier shard.
        const auto it = std::lower_bound(cum.begin(), cum.end(), target);
        const int64_t cut = static_cast<int64_t>(it - cum.begin()) + 1;
        bounds[k] = static_cast<int32_t>(std::min<int64_t>(cut, n_rows));
    }
    bounds[n_shards] = n_rows;
    for (int32_t k = 1; k <= n_shards; ++k) bounds[k] = std::max(bounds[k], bounds[k - 1]);
}

// Per-shard scale of the rebalancing cut: measured time / modelled weight
// (1 for a shard without weight).
std::vector<double> shard_scales(const int32_t* rowoff, double edge_w, double store_w,
                                 int32_t n_shards, const int32_t* old_bounds,
                                 const double* shard_time) {
    std::vector<double> scale(static_cast<size_t>(n_shards), 1.0);
    for (int32_t g = 0; g < n_shards; ++g) {
        double W = 0.0;
        for (int32_t r = old_bounds[g]; r < old_bounds[g + 1]; ++r) {
            const double deg = static_cast<double>(static_cast<int64_t>(rowoff[r + 1]) - rowoff[r]);
            W = W + (deg * edge_w + store_w);
        }
        if (W > 0.0) {
            need(shard_time[g] > 0.0 && std::isfinite(shard_time[g]), CWLB_ERR_INVALID_ARGUMENT,
                 "shard times must be positive and finite");
            scale[static_cast<size_t>(g)] = shard_time[g] / W;
        }
    }
    return scale;
}

__global__ void rebase_offsets_kernel(const int32_t* __restrict__ in, int64_t count, int32_t base,
                                      int32_t* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) out[i] = in[i] - base;
}

void validate_offsets(int32_t n_rows, int32_t nnz, const int32_t* rowoff) {
    need(rowoff[0] == 0, CWLB_ERR_INVALID_ARGUMENT, "row_offset[0] must be 0");
    need(rowoff[n_rows] == nnz, CWLB_ERR_RUNTIME,
         "Inconsistent NNZ count: row_offset[rows] != nnz");
    for (int32_t r = 0; r < n_rows; ++r)
        need(rowoff[r + 1] >= rowoff[r], CWLB_ERR_INVALID_ARGUMENT,
             "row offsets are not monotone");
}

// Sort, partition and check the shard's block; `d_rowoff_local` holds the
// block's rebased offsets (n + 1), `d_col` / `d_val` its nonzeros.
void build_shard(cwlb_shard* sh, const int32_t* d_rowoff_local, const int32_t* d_col,
                 const float* d_val, const cwlb_costs& costs, double capacity) {
    cwlb_ctx* ctx = sh->ctx;
    const size_t n = static_cast<size_t>(sh->n), nnz = static_cast<size_t>(sh->nnz);
    int32_t* org = sh->origin.as<int32_t>(std::max<size_t>(n, 1));
    int32_t* sro = sh->rowoff.as<int32_t>(n + 1);
    int32_t* scol = sh->col.as<int32_t>(std::max<size_t>(nnz, 1));
    float* sval = sh->val.as<float>(std::max<size_t>(nnz, 1));
    if (sh->n == 0) {
        CWLB_CUDA(cudaMemsetAsync(sro, 0, sizeof(int32_t), ctx->stream));
        return;
    }
    launch_sort_by_degree(ctx, sh->n, sh->nnz, d_rowoff_local, d_col, d_val, org, sro, scol, sval);
    if (sh->nnz > 0) {
        DeviceBuffer flag;
        sh->unit = values_all_one(ctx, sval, nnz,
                                  static_cast<unsigned int*>(flag.ensure(sizeof(unsigned int))));
    }
    const int64_t cnt = run_partition(ctx, sh->n, sro, costs, capacity);
    sh->segment = cwlb_segment_size(&costs, capacity);
    sh->n_tasks = cnt;
    if (cnt > 0) {
        cwlb_task* t = sh->tasks.as<cwlb_task>(static_cast<size_t>(cnt));
        CWLB_CUDA(cudaMemcpyAsync(t, ctx->part_tasks.ptr, sizeof(cwlb_task) * cnt,
                                  cudaMemcpyDeviceToDevice, ctx->stream));
        int64_t bad = 0, unc = 0, nz = 0;
        run_tasks_check(ctx, sh->n, sh->nnz, sro, t, cnt, &bad, &unc, &nz);
        if (bad == 0 && unc == 0 && nz == 0) sh->flags = CWLB_ROWS_COVERED;
    }
    CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
}

cwlb_shard* new_shard(cwlb_ctx* ctx, int32_t shard, int32_t n_shards, const int32_t* bounds,
                      const int32_t* h_rowoff) {
    auto* sh = new cwlb_shard();
    sh->ctx = ctx;
    sh->shard = shard;
    sh->n_shards = n_shards;
    sh->row_begin = bounds[shard];
    sh->row_end = bounds[shard + 1];
    sh->n = sh->row_end - sh->row_begin;
    sh->nnz = h_rowoff[sh->row_end] - h_rowoff[sh->row_begin];
    return sh;
}

void free_shard(cwlb_shard* sh) {
    if (!sh) return;
    if (sh->ctx) cudaSetDevice(sh->ctx->device);
    for (DeviceBuffer* b : {&sh->origin, &sh->rowoff, &sh->col, &sh->val, &sh->tasks}) b->release();
    delete sh;
}

void check_shard_args(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const cwlb_costs* costs,
                      int32_t shard, int32_t n_shards, cwlb_shard** out) {
    need(ctx != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null context");
    need(out != nullptr && costs != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null argument");
    need(n_rows >= 0 && nnz >= 0, CWLB_ERR_INVALID_ARGUMENT, "negative size");
    need(n_shards >= 1 && shard >= 0 && shard < n_shards, CWLB_ERR_INVALID_ARGUMENT,
         "shard index outside [0, n_shards)");
}

// The cut of a shard build: `cut` checked and copied, or (NULL) the modelled
// cut of cwlb_shard_bounds.
std::vector<int32_t> build_cut(int32_t n_rows, const int32_t* rowoff, const cwlb_costs& costs,
                               const int32_t* cut, int32_t n_shards) {
    std::vector<int32_t> bounds(static_cast<size_t>(n_shards) + 1);
    if (cut) {
        need(cut[0] == 0 && cut[n_shards] == n_rows, CWLB_ERR_INVALID_ARGUMENT,
             "cut must start at 0 and end at n_rows");
        for (int32_t g = 0; g < n_shards; ++g)
            need(cut[g] <= cut[g + 1], CWLB_ERR_INVALID_ARGUMENT, "cut must be non-decreasing");
        std::copy(cut, cut + n_shards + 1, bounds.begin());
    } else {
        shard_bounds_host(n_rows, rowoff, costs.C_compute_ns + costs.C_load_ns, costs.C_store_ns,
                          n_shards, bounds.data());
    }
    return bounds;
}

cwlb_shard* shard_create_host(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                              const int32_t* col, const float* val, const cwlb_costs& costs,
                              double capacity, int32_t shard, int32_t n_shards,
                              const int32_t* cut = nullptr) {
    CWLB_CUDA(cudaSetDevice(ctx->device));
    validate_offsets(n_rows, nnz, rowoff);
    const std::vector<int32_t> bounds = build_cut(n_rows, rowoff, costs, cut, n_shards);
    cwlb_shard* sh = new_shard(ctx, shard, n_shards, bounds.data(), rowoff);
    try {
        const int32_t e0 = rowoff[sh->row_begin];
        std::vector<int32_t> local(static_cast<size_t>(sh->n) + 1);
        for (int32_t i = 0; i <= sh->n; ++i) local[static_cast<size_t>(i)] = rowoff[sh->row_begin + i] - e0;
        int32_t* d_ro = ctx->in_rowoff.as<int32_t>(local.size());
        int32_t* d_col = ctx->in_col.as<int32_t>(std::max<size_t>(sh->nnz, 1));
        float* d_val = ctx->in_val.as<float>(std::max<size_t>(sh->nnz, 1));
        copy_to_device(ctx, d_ro, local.data(), sizeof(int32_t) * local.size(), ctx->stream);
        if (sh->nnz > 0) {
            copy_to_device(ctx, d_col, col + e0, sizeof(int32_t) * sh->nnz, ctx->stream);
            copy_to_device(ctx, d_val, val + e0, sizeof(float) * sh->nnz, ctx->stream);
        }
        build_shard(sh, d_ro, d_col, d_val, costs, capacity);
    } catch (...) {
        free_shard(sh);
        throw;
    }
    return sh;
}

// Aggregation of a built shard into d_out (rows [0, n) = original rows
// [row_begin, row_end)); asynchronous on the context's stream.
void shard_aggregate(cwlb_shard* sh, const float* d_H, int64_t h_rows, int64_t K, float* d_out,
                     uint32_t flags) {
    need(K >= 0 && h_rows >= 0, CWLB_ERR_INVALID_ARGUMENT, "negative size");
    need(sh->n == 0 || K == 0 || ((d_H != nullptr || h_rows == 0) && d_out != nullptr),
         CWLB_ERR_INVALID_ARGUMENT, "null device buffer");
    need((flags & ~static_cast<uint32_t>(CWLB_DETERMINISTIC)) == 0, CWLB_ERR_INVALID_ARGUMENT,
         "unknown flags (only CWLB_DETERMINISTIC applies to a shard)");
    CWLB_CUDA(cudaSetDevice(sh->ctx->device));
    if (sh->n == 0 || K == 0) return;
    launch_spmm_mean(sh->ctx, sh->n, sh->nnz, sh->rowoff.as<int32_t>(0), sh->col.as<int32_t>(0),
                     sh->unit ? nullptr : sh->val.as<float>(0), sh->origin.as<int32_t>(0), d_H,
                     h_rows, K,
                     sh->tasks.as<cwlb_task>(0), sh->n_tasks, d_out, sh->flags | flags);
}

uint32_t take_errors(cwlb_ctx* ctx) {
    uint32_t flags = 0;
    CWLB_CUDA(cudaMemcpyAsync(&flags, ctx->d_error_flags, sizeof(flags), cudaMemcpyDeviceToHost,
                              ctx->stream));
    CWLB_CUDA(cudaMemsetAsync(ctx->d_error_flags, 0, sizeof(uint32_t), ctx->stream));
    CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
    return flags;
}

void enable_peers(cwlb_ctx* const* ctxs, int32_t n) {
    for (int32_t d = 0; d < n; ++d) {
        CWLB_CUDA(cudaSetDevice(ctxs[d]->device));
        for (int32_t s = 0; s < n; ++s) {
            if (s == d || ctxs[s]->device == ctxs[d]->device) continue;
            int ok = 0;
            CWLB_CUDA(cudaDeviceCanAccessPeer(&ok, ctxs[d]->device, ctxs[s]->device));
            if (!ok) continue;  // cudaMemcpyPeerAsync still works, through the host
            const cudaError_t e = cudaDeviceEnablePeerAccess(ctxs[s]->device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) {
                cudaGetLastError();
            } else {
                CWLB_CUDA(e);
            }
        }
    }
}

}  // namespace
}  // namespace cwlb

extern "C" {

int cwlb_shard_bounds(int32_t n_rows, const int32_t* row_offset, const cwlb_costs* costs,
                      int32_t n_shards, int32_t* bounds) {
    return cwlb::guarded_multi([&] {
        cwlb::need(costs && bounds && (n_rows == 0 || row_offset), CWLB_ERR_INVALID_ARGUMENT,
                   "null argument");
        cwlb::need(n_rows >= 0 && n_shards >= 1, CWLB_ERR_INVALID_ARGUMENT,
                   "n_rows must be >= 0 and n_shards >= 1");
        if (n_rows == 0) {
            std::fill(bounds, bounds + n_shards + 1, 0);
            return;
        }
        cwlb::shard_bounds_host(n_rows, row_offset, costs->C_compute_ns + costs->C_load_ns,
                                costs->C_store_ns, n_shards, bounds);
    });
}

int cwlb_shard_bounds_rebalance(int32_t n_rows, const int32_t* row_offset,
                                const cwlb_costs* costs, int32_t n_shards,
                                const int32_t* bounds, const double* shard_time,
                                int32_t* new_bounds) {
    return cwlb::guarded_multi([&] {
        cwlb::need(costs && bounds && shard_time && new_bounds && (n_rows == 0 || row_offset),
                   CWLB_ERR_INVALID_ARGUMENT, "null argument");
        cwlb::need(n_rows >= 0 && n_shards >= 1, CWLB_ERR_INVALID_ARGUMENT,
                   "n_rows must be >= 0 and n_shards >= 1");
        cwlb::need(bounds[0] == 0 && bounds[n_shards] == n_rows, CWLB_ERR_INVALID_ARGUMENT,
                   "bounds must start at 0 and end at n_rows");
        for (int32_t g = 0; g < n_shards; ++g)
            cwlb::need(bounds[g] <= bounds[g + 1], CWLB_ERR_INVALID_ARGUMENT,
                       "bounds must be non-decreasing");
        if (n_rows == 0) {
            std::fill(new_bounds, new_bounds + n_shards + 1, 0);
            return;
        }
        const double ew = costs->C_compute_ns + costs->C_load_ns, sw = costs->C_store_ns;
        const std::vector<double> scale =
            cwlb::shard_scales(row_offset, ew, sw, n_shards, bounds, shard_time);
        std::vector<int32_t> nb(static_cast<size_t>(n_shards) + 1);  // bounds may alias
        cwlb::shard_bounds_host(n_rows, row_offset, ew, sw, n_shards, nb.data(), bounds,
                                scale.data());
        std::copy(nb.begin(), nb.end(), new_bounds);
    });
}

int cwlb_shard_create(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                      const int32_t* col_ind, const float* value, const cwlb_costs* costs,
                      double capacity, int32_t shard, int32_t n_shards, cwlb_shard** out) {
    return cwlb_shard_create_cut(ctx, n_rows, nnz, row_offset, col_ind, value, costs, capacity,
                                 nullptr, shard, n_shards, out);
}

int cwlb_shard_create_cut(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* row_offset,
                          const int32_t* col_ind, const float* value, const cwlb_costs* costs,
                          double capacity, const int32_t* cut, int32_t shard, int32_t n_shards,
                          cwlb_shard** out) {
    return cwlb::guarded_multi([&] {
        cwlb::check_shard_args(ctx, n_rows, nnz, costs, shard, n_shards, out);
        *out = nullptr;
        cwlb::need(row_offset && (nnz == 0 || (col_ind && value)), CWLB_ERR_INVALID_ARGUMENT,
                   "null host buffer");
        *out = cwlb::shard_create_host(ctx, n_rows, nnz, row_offset, col_ind, value, *costs,
                                       capacity, shard, n_shards, cut);
    });
}

int cwlb_shard_create_device(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                             const int32_t* d_row_offset, const int32_t* d_col_ind,
                             const float* d_value, const cwlb_costs* costs, double capacity,
                             int32_t shard, int32_t n_shards, cwlb_shard** out) {
    return cwlb_shard_create_device_cut(ctx, n_rows, nnz, d_row_offset, d_col_ind, d_value, costs,
                                        capacity, nullptr, shard, n_shards, out);
}

int cwlb_shard_create_device_cut(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz,
                                 const int32_t* d_row_offset, const int32_t* d_col_ind,
                                 const float* d_value, const cwlb_costs* costs, double capacity,
                                 const int32_t* cut, int32_t shard, int32_t n_shards,
                                 cwlb_shard** out) {
    return cwlb::guarded_multi([&] {
        cwlb::check_shard_args(ctx, n_rows, nnz, costs, shard, n_shards, out);
        *out = nullptr;
        cwlb::need(d_row_offset && (nnz == 0 || (d_col_ind && d_value)),
                   CWLB_ERR_INVALID_ARGUMENT, "null device buffer");
        CWLB_CUDA(cudaSetDevice(ctx->device));
        // The cut points need the offsets on the host (4 (rows + 1) bytes).
        std::vector<int32_t> h(static_cast<size_t>(n_rows) + 1);
        CWLB_CUDA(cudaMemcpyAsync(h.data(), d_row_offset, sizeof(int32_t) * h.size(),
                                  cudaMemcpyDeviceToHost, ctx->stream));
        CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
        cwlb::validate_offsets(n_rows, nnz, h.data());
        const std::vector<int32_t> bounds = cwlb::build_cut(n_rows, h.data(), *costs, cut, n_shards);
        cwlb_shard* sh = cwlb::new_shard(ctx, shard, n_shards, bounds.data(), h.data());
        try {
            const int32_t e0 = h[static_cast<size_t>(sh->row_begin)];
            int32_t* d_ro = ctx->in_rowoff.as<int32_t>(static_cast<size_t>(sh->n) + 1);
            const int64_t cnt = static_cast<int64_t>(sh->n) + 1;
            cwlb::rebase_offsets_kernel<<<static_cast<unsigned>(cwlb::ceil_div(cnt, 256)), 256, 0,
                                          ctx->stream>>>(d_row_offset + sh->row_begin, cnt, e0, d_ro);
            CWLB_LAUNCH_CHECK("rebase_offsets_kernel");
            cwlb::build_shard(sh, d_ro, d_col_ind + e0, d_value + e0, *costs, capacity);
        } catch (...) {
            cwlb::free_shard(sh);
            throw;
        }
        *out = sh;
    });
}

int cwlb_shard_info(const cwlb_shard* sh, int32_t* row_begin, int32_t* row_end, int32_t* nnz,
                    int64_t* n_tasks, int32_t* segment_size) {
    return cwlb::guarded_multi([&] {
        cwlb::need(sh != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null shard");
        if (row_begin) *row_begin = sh->row_begin;
        if (row_end) *row_end = sh->row_end;
        if (nnz) *nnz = sh->nnz;
        if (n_tasks) *n_tasks = sh->n_tasks;
        if (segment_size) *segment_size = sh->segment;
    });
}

int cwlb_shard_tasks(const cwlb_shard* sh, const cwlb_task** d_tasks) {
    return cwlb::guarded_multi([&] {
        cwlb::need(sh != nullptr && d_tasks != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null argument");
        *d_tasks = static_cast<const cwlb_task*>(sh->tasks.ptr);
    });
}

int cwlb_shard_aggregate_device(cwlb_shard* sh, const float* d_H, int64_t h_rows, int64_t K,
                                float* d_out, uint32_t flags) {
    return cwlb::guarded_multi([&] {
        cwlb::need(sh != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null shard");
        cwlb::shard_aggregate(sh, d_H, h_rows, K, d_out, flags);
    });
}

int cwlb_shard_destroy(cwlb_shard* sh) {
    return cwlb::guarded_multi([&] { cwlb::free_shard(sh); });
}

int cwlb_spmm_mean_multi(cwlb_ctx* const* ctxs, int32_t n_gpus, int32_t n_rows, int32_t nnz,
                         const int32_t* row_offset, const int32_t* col_ind, const float* value,
                         const float* H, int64_t h_rows, int64_t K, const cwlb_costs* costs,
                         double capacity, float* out, double* time_us) {
    return cwlb::guarded_multi([&] {
        cwlb::need(ctxs != nullptr && n_gpus >= 1, CWLB_ERR_INVALID_ARGUMENT,
                   "need at least one context");
        for (int32_t g = 0; g < n_gpus; ++g)
            cwlb::need(ctxs[g] != nullptr, CWLB_ERR_INVALID_ARGUMENT, "null context");
        for (int32_t a = 0; a < n_gpus; ++a)
            for (int32_t b = a + 1; b < n_gpus; ++b)
                cwlb::need(ctxs[a] != ctxs[b], CWLB_ERR_INVALID_ARGUMENT,
                           "a context may appear only once (one host thread each)");
        cwlb::need(costs && row_offset && (nnz == 0 || (col_ind && value)),
                   CWLB_ERR_INVALID_ARGUMENT, "null argument");
        cwlb::need(n_rows >= 0 && nnz >= 0 && h_rows >= 0 && K >= 0, CWLB_ERR_INVALID_ARGUMENT,
                   "negative size");
        cwlb::need(n_rows == 0 || K == 0 || (out && (H || h_rows == 0)),
                   CWLB_ERR_INVALID_ARGUMENT, "null argument");
        if (time_us) *time_us = 0.0;
        cwlb::validate_offsets(n_rows, nnz, row_offset);
        if (n_rows == 0 || K == 0) {
            if (out && n_rows > 0) std::fill(out, out + static_cast<size_t>(n_rows) * K, 0.0f);
            return;
        }
        std::vector<int> codes(static_cast<size_t>(n_gpus), CWLB_OK);
        std::vector<std::string> msgs(static_cast<size_t>(n_gpus));
        std::vector<double> us(static_cast<size_t>(n_gpus), 0.0);
        auto work = [&](int32_t g) {
            cwlb_ctx* ctx = ctxs[g];
            cwlb_shard* sh = nullptr;
            try {
                CWLB_CUDA(cudaSetDevice(ctx->device));
                sh = cwlb::shard_create_host(ctx, n_rows, nnz, row_offset, col_ind, value,
                                             *costs, capacity, g, n_gpus);
                if (sh->n > 0) {
                    const size_t hb = sizeof(float) * static_cast<size_t>(h_rows) * K;
                    float* d_H = ctx->in_H.as<float>(std::max<size_t>(hb / sizeof(float), 1));
                    if (hb) cwlb::copy_to_device(ctx, d_H, H, hb, ctx->stream);
                    const size_t ob = sizeof(float) * static_cast<size_t>(sh->n) * K;
                    float* d_out = ctx->out_buf.as<float>(ob / sizeof(float));
                    CWLB_CUDA(cudaEventRecord(ctx->ev_start, ctx->stream));
                    cwlb::shard_aggregate(sh, d_H, h_rows, K, d_out, 0);
                    CWLB_CUDA(cudaEventRecord(ctx->ev_stop, ctx->stream));
                    cwlb::copy_to_host(ctx, out + static_cast<size_t>(sh->row_begin) * K, d_out, ob,
                                       ctx->stream);
                    CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
                    float ms = 0.0f;
                    CWLB_CUDA(cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop));
                    us[static_cast<size_t>(g)] = 1e3 * ms;
                    const uint32_t e = cwlb::take_errors(ctx);
                    if (e) cwlb::fail(CWLB_ERR_INVALID_ARGUMENT,
                                      "invalid input detected on the device (flags " +
                                          std::to_string(e) + ")");
                }
            } catch (const cwlb::Failure& e) {
                codes[static_cast<size_t>(g)] = e.code;
                msgs[static_cast<size_t>(g)] = e.what();
            } catch (const std::bad_alloc&) {
                codes[static_cast<size_t>(g)] = CWLB_ERR_OUT_OF_MEMORY;
                msgs[static_cast<size_t>(g)] = "host allocation failed";
            } catch (const std::exception& e) {
                codes[static_cast<size_t>(g)] = CWLB_ERR_RUNTIME;
                msgs[static_cast<size_t>(g)] = e.what();
            }
            cwlb::free_shard(sh);
        };
        std::vector<std::thread> pool;
        for (int32_t g = 1; g < n_gpus; ++g) pool.emplace_back(work, g);
        work(0);
        for (auto& t : pool) t.join();
        for (int32_t g = 0; g < n_gpus; ++g) {
            if (codes[static_cast<size_t>(g)] != CWLB_OK) {
                cwlb::fail(codes[static_cast<size_t>(g)],
                           "GPU " + std::to_string(ctxs[g]->device) + " (shard " +
                               std::to_string(g) + "): " + msgs[static_cast<size_t>(g)]);
            }
        }
        if (time_us) *time_us = *std::max_element(us.begin(), us.end());
    });
}

int cwlb_gather_rows_multi(cwlb_ctx* const* ctxs, int32_t n_gpus, float* const* d_X,
                           int64_t rows, int64_t K, const int32_t* bounds) {
    return cwlb::guarded_multi([&] {
        cwlb::need(ctxs && d_X && bounds && n_gpus >= 1, CWLB_ERR_INVALID_ARGUMENT,
                   "null argument");
        cwlb::need(rows >= 0 && K >= 0, CWLB_ERR_INVALID_ARGUMENT, "negative size");
        cwlb::need(bounds[0] == 0 && bounds[n_gpus] == rows, CWLB_ERR_INVALID_ARGUMENT,
                   "bounds must start at 0 and end at rows");
        for (int32_t g = 0; g < n_gpus; ++g) {
            cwlb::need(ctxs[g] && d_X[g], CWLB_ERR_INVALID_ARGUMENT, "null context or buffer");
            cwlb::need(bounds[g + 1] >= bounds[g], CWLB_ERR_INVALID_ARGUMENT,
                       "bounds must not decrease");
        }
        if (n_gpus == 1 || rows == 0 || K == 0) return;
        cwlb::enable_peers(ctxs, n_gpus);
        // Every source block is complete once its owner's stream reaches
        // this point; each destination stream waits for every source, copies
        // the blocks in, and every stream then waits for every destination's
        // copies, so later work on any context's stream sees the full matrix
        // everywhere and no source is overwritten while it is being read.
        std::vector<cudaEvent_t> ready(static_cast<size_t>(n_gpus)), done(static_cast<size_t>(n_gpus));
        for (int32_t g = 0; g < n_gpus; ++g) {
            CWLB_CUDA(cudaSetDevice(ctxs[g]->device));
            CWLB_CUDA(cudaEventCreateWithFlags(&ready[g], cudaEventDisableTiming));
            CWLB_CUDA(cudaEventCreateWithFlags(&done[g], cudaEventDisableTiming));
            CWLB_CUDA(cudaEventRecord(ready[g], ctxs[g]->stream));
        }
        for (int32_t d = 0; d < n_gpus; ++d) {
            CWLB_CUDA(cudaSetDevice(ctxs[d]->device));
            for (int32_t s = 0; s < n_gpus; ++s) {
                if (s == d || bounds[s + 1] == bounds[s]) continue;
                CWLB_CUDA(cudaStreamWaitEvent(ctxs[d]->stream, ready[s], 0));
                const size_t off = static_cast<size_t>(bounds[s]) * K;
                const size_t bytes = sizeof(float) * static_cast<size_t>(bounds[s + 1] - bounds[s]) * K;
                CWLB_CUDA(cudaMemcpyPeerAsync(d_X[d] + off, ctxs[d]->device, d_X[s] + off,
                                              ctxs[s]->device, bytes, ctxs[d]->stream));
            }
            CWLB_CUDA(cudaEventRecord(done[d], ctxs[d]->stream));
        }
        for (int32_t g = 0; g < n_gpus; ++g) {
            CWLB_CUDA(cudaSetDevice(ctxs[g]->device));
            for (int32_t d = 0; d < n_gpus; ++d)
                if (d != g) CWLB_CUDA(cudaStreamWaitEvent(ctxs[g]->stream, done[d], 0));
        }
        for (int32_t g = 0; g < n_gpus; ++g) {
            CWLB_CUDA(cudaSetDevice(ctxs[g]->device));
            cudaEventDestroy(ready[g]);
            cudaEventDestroy(done[g]);
        }
    });
}

}  // extern "C"
