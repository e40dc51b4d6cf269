// C bridge over the CWLB-SpMM reference, compiled from its unmodified sources
// (main.cpp, weightCost.cpp, src/*.cpp) against the host stand-ins in
// oracle/shim/.  TEST INFRASTRUCTURE ONLY: the product library never links
// it; tests and tests/golden/gen_golden.py load oracle/_ref/libcwlbref.so to
// pin the oracle and to produce golden fixtures.
//
// Every function returns 0 on success, or 1 (std::invalid_argument),
// 2 (std::runtime_error), 3 (std::overflow_error), 4 (other exception), with
// the exception text available from cwlbref_last_error().
#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "Matrix.h"
#include "config.h"
#include "data.h"
#include "parallelMatrix.h"
#include "utils.h"

// Functions with external linkage defined in the reference's main.cpp
// (compiled with -Dmain=cwlb_reference_main) and weightCost.cpp.
std::array<int, 3> recommended_candidate_w(std::uint64_t nnz);
std::pair<int, int> candidate_search_bounds(const std::array<int, 3>& values, std::size_t best_index);
std::vector<int> candidate_search_by_count(int lower, int upper, int requested);
std::vector<int> candidate_search_by_step(int lower, int upper, int step);
int positive_search_argument(const std::string& text);
CSR_Order sortCSRByDegreeDPLCPU(const CSR& csr);
double capacity_from_s(int s, const SpmmCostParams& costs);
int wave_based_s(const CSR_Order& sorted_csr, int compute_units, int wave);
Defined::RowMajorMatrixXf deterministic_features(int rows, int cols);
int cwlb_reference_main(int argc, char* argv[]);
int cwlb_costwrite_main(int argc, char* argv[]);

namespace {
std::string g_err;
std::vector<ParallelDataWeighted> g_tasks;
CSR g_loaded;

template <typename F>
int guarded(F&& f) {
    try {
        f();
        g_err.clear();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return 1;
    } catch (const std::overflow_error& e) {
        g_err = e.what();
        return 3;
    } catch (const std::runtime_error& e) {
        g_err = e.what();
        return 2;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 4;
    }
}

SpmmCostParams costs_from(const double* c) {
    SpmmCostParams p;
    p.C_compute_ns = c[0];
    p.C_load_ns = c[1];
    p.C_store_ns = c[2];
    p.C_atomic_ns = c[3];
    return p;
}

CSR_Order order_from(int n_rows, int nnz, const int* rowoff, const int* col,
                     const float* val, const int* origin) {
    CSR_Order o;
    o.RowOffset.assign(rowoff, rowoff + n_rows + 1);
    o.ColInd.assign(col, col + nnz);
    o.Value.assign(val, val + nnz);
    o.Origin_local.assign(origin, origin + n_rows);
    return o;
}
}  // namespace

extern "C" {

const char* cwlbref_last_error() { return g_err.c_str(); }

void cwlbref_set_device(long max_wg, long sub_group, long local_mem, long compute_units) {
    auto& t = sycl::detail::device_table();
    t.max_work_group_size = static_cast<std::size_t>(max_wg);
    t.sub_group_sizes = {static_cast<std::size_t>(sub_group)};
    t.local_mem_size = static_cast<std::uint64_t>(local_mem);
    t.max_compute_units = static_cast<std::uint32_t>(compute_units);
}

// main.cpp:197-278
int cwlbref_sort_by_degree(int n_rows, int nnz, const int* rowoff, const int* col,
                           const float* val, int* origin, int* new_rowoff,
                           int* new_col, float* new_val) {
    return guarded([&] {
        CSR csr;
        csr.RowOffset.assign(rowoff, rowoff + n_rows + 1);
        csr.ColInd.assign(col, col + nnz);
        csr.Value.assign(val, val + nnz);
        const CSR_Order o = sortCSRByDegreeDPLCPU(csr);
        std::copy(o.Origin_local.begin(), o.Origin_local.end(), origin);
        std::copy(o.RowOffset.begin(), o.RowOffset.end(), new_rowoff);
        std::copy(o.ColInd.begin(), o.ColInd.end(), new_col);
        std::copy(o.Value.begin(), o.Value.end(), new_val);
    });
}

// src/utils.cpp:832-1021.  Stores the task list; fetch it with
// cwlbref_partition_fetch.
int cwlbref_partition(int n_rows, const int* rowoff, const double* costs, double capacity,
                      std::int64_t* n_tasks) {
    return guarded([&] {
        CSR_Order o;
        o.RowOffset.assign(rowoff, rowoff + n_rows + 1);
        g_tasks = costWeightedTaskPartitioning(o, costs_from(costs), capacity);
        *n_tasks = static_cast<std::int64_t>(g_tasks.size());
    });
}

void cwlbref_partition_fetch(int* out) {
    static_assert(sizeof(ParallelDataWeighted) == 4 * sizeof(int), "task layout");
    if (!g_tasks.empty()) std::memcpy(out, g_tasks.data(), g_tasks.size() * sizeof(ParallelDataWeighted));
}

// src/parallelMatrix.cpp:63-254 (large_k == 0) or :264-683 (large_k != 0).
int cwlbref_spmm(int large_k, int n_rows, int nnz, const int* rowoff, const int* col,
                 const float* val, const int* origin, const float* H, long h_rows, long K,
                 int dim_hint, int local_dimension, const int* tasks, long n_tasks,
                 float* out, double* time_us) {
    return guarded([&] {
        const CSR_Order o = order_from(n_rows, nnz, rowoff, col, val, origin);
        Defined::RowMajorMatrixXf h(h_rows, K);
        if (h_rows * K) std::memcpy(h.data(), H, sizeof(float) * h_rows * K);
        std::vector<ParallelDataWeighted> t(static_cast<std::size_t>(n_tasks));
        if (n_tasks) std::memcpy(t.data(), tasks, sizeof(ParallelDataWeighted) * n_tasks);
        sycl::queue q;
        double time = -1.0;
        Defined::RowMajorMatrixXf c =
            large_k ? spmmKernelLargeKFallback(q, o, h, dim_hint, local_dimension, t, time)
                    : spmmKernel(q, o, h, dim_hint, local_dimension, t, time);
        if (c.rows() * c.cols()) std::memcpy(out, c.data(), sizeof(float) * c.rows() * c.cols());
        *time_us = time;
    });
}

// main.cpp:281-292
double cwlbref_capacity_from_s(int s, const double* costs) {
    return capacity_from_s(s, costs_from(costs));
}

// main.cpp:295-321
int cwlbref_wave_based_s(int n_rows, const int* rowoff, int compute_units, int wave, int* s) {
    return guarded([&] {
        CSR_Order o;
        if (n_rows >= 0 && rowoff) o.RowOffset.assign(rowoff, rowoff + n_rows + 1);
        *s = wave_based_s(o, compute_units, wave);
    });
}

// main.cpp:87-95
void cwlbref_recommended_w(std::uint64_t nnz, int* out) {
    const auto w = recommended_candidate_w(nnz);
    out[0] = w[0];
    out[1] = w[1];
    out[2] = w[2];
}

// main.cpp:109-127
int cwlbref_search_bounds(const int* values, long best_index, int* out) {
    return guarded([&] {
        const auto b = candidate_search_bounds({values[0], values[1], values[2]},
                                               static_cast<std::size_t>(best_index));
        out[0] = b.first;
        out[1] = b.second;
    });
}

// main.cpp:130-167 (by_step != 0 selects candidate_search_by_step).
int cwlbref_search_grid(int by_step, int lower, int upper, int arg, int* out, int max_out,
                        int* n_out) {
    return guarded([&] {
        const auto v = by_step ? candidate_search_by_step(lower, upper, arg)
                               : candidate_search_by_count(lower, upper, arg);
        *n_out = static_cast<int>(v.size());
        for (int i = 0; i < static_cast<int>(v.size()) && i < max_out; ++i) out[i] = v[i];
    });
}

// main.cpp:99-106
int cwlbref_positive_search_argument(const char* text, int* value) {
    return guarded([&] { *value = positive_search_argument(text); });
}

// main.cpp:324-336
void cwlbref_features(int rows, int cols, float* out) {
    const auto f = deterministic_features(rows, cols);
    if (static_cast<long>(rows) * cols) std::memcpy(out, f.data(), sizeof(float) * rows * cols);
}

// src/utils.cpp:1024-1075
int cwlbref_save_costs(const double* costs, const char* path, int append, int precision) {
    return save_costs_one_per_line(costs_from(costs), path, append != 0, precision) ? 0 : 2;
}

// src/utils.cpp:1077-1092
int cwlbref_read_costs(double* costs, const char* path) {
    SpmmCostParams p;
    if (!read_costs_one_per_line(p, path)) return 2;
    costs[0] = p.C_compute_ns;
    costs[1] = p.C_load_ns;
    costs[2] = p.C_store_ns;
    costs[3] = p.C_atomic_ns;
    return 0;
}

// src/data.cpp:121-130.  The path is resolved against "../resources/datasets/"
// relative to the working directory, as in the reference.
int cwlbref_load_csr(const char* name, int* V, int* E) {
    return guarded([&] { g_loaded = loadDatasetToCSR(name, *V, *E); });
}

void cwlbref_load_csr_fetch(int* rowoff, int* col, float* val) {
    std::copy(g_loaded.RowOffset.begin(), g_loaded.RowOffset.end(), rowoff);
    std::copy(g_loaded.ColInd.begin(), g_loaded.ColInd.end(), col);
    std::copy(g_loaded.Value.begin(), g_loaded.Value.end(), val);
}

// src/utils.cpp:1117-1265 (returns 1 when the comparison passes).
int cwlbref_validate(const float* result, const float* reference, long rows, long cols,
                     int n_rows, int nnz, const int* rowoff, const int* col, const float* val,
                     const float* dense, long dense_rows, float abs_tol) {
    Defined::RowMajorMatrixXf r(rows, cols), ref(rows, cols), d(dense_rows, cols);
    if (rows * cols) {
        std::memcpy(r.data(), result, sizeof(float) * rows * cols);
        std::memcpy(ref.data(), reference, sizeof(float) * rows * cols);
    }
    if (dense_rows * cols) std::memcpy(d.data(), dense, sizeof(float) * dense_rows * cols);
    CSR csr;
    csr.RowOffset.assign(rowoff, rowoff + n_rows + 1);
    csr.ColInd.assign(col, col + nnz);
    csr.Value.assign(val, val + nnz);
    return validate_custom_csr_result(r, ref, csr, d, abs_tol) ? 1 : 0;
}

// src/utils.cpp:1117-1265 with independent shapes for the result, the
// reference and the dense matrix, and the CSR given by its RowOffset length
// (the shape checks need all of them).  Returns 1 when the comparison passes.
int cwlbref_validate_shapes(const float* result, long rr, long rc, const float* reference,
                            long fr, long fc, const int* rowoff, long rowoff_len, const int* col,
                            long nnz, const float* val, const float* dense, long dr, long dc,
                            float abs_tol) {
    Defined::RowMajorMatrixXf r(rr, rc), ref(fr, fc), d(dr, dc);
    if (rr * rc) std::memcpy(r.data(), result, sizeof(float) * rr * rc);
    if (fr * fc) std::memcpy(ref.data(), reference, sizeof(float) * fr * fc);
    if (dr * dc) std::memcpy(d.data(), dense, sizeof(float) * dr * dc);
    CSR csr;
    csr.RowOffset.assign(rowoff, rowoff + rowoff_len);
    csr.ColInd.assign(col, col + nnz);
    csr.Value.assign(val, val + nnz);
    return validate_custom_csr_result(r, ref, csr, d, abs_tol) ? 1 : 0;
}

// weightCost.cpp / src/utils.cpp:342-829 run on the emulated device.
int cwlbref_measure_costs(int K, int repeat, int WI, int load_mb, int writers, double* out) {
    return guarded([&] {
        sycl::queue q;
        const SpmmCostParams p = measure_spmm_costs(q, K, repeat, WI, load_mb, writers);
        out[0] = p.C_compute_ns;
        out[1] = p.C_load_ns;
        out[2] = p.C_store_ns;
        out[3] = p.C_atomic_ns;
    });
}

int cwlbref_main(int argc, char** argv) { return cwlb_reference_main(argc, argv); }
int cwlbref_costwrite_main(int argc, char** argv) { return cwlb_costwrite_main(argc, argv); }

}  // extern "C"
