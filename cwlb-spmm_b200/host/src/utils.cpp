// Interface functions of include/utils.h over libcwlb_spmm.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <iomanip>
#include <iostream>
#include <limits>
#include <stdexcept>

#include "utils.h"

static_assert(sizeof(ParallelDataWeighted) == sizeof(cwlb_task), "task layout");

namespace {
cwlb_costs to_c(const SpmmCostParams& p) {
    cwlb_costs c{};
    c.C_compute_ns = p.C_compute_ns;
    c.C_load_ns = p.C_load_ns;
    c.C_store_ns = p.C_store_ns;
    c.C_atomic_ns = p.C_atomic_ns;
    c.K = p.K;
    c.WI = p.WI;
    c.repeat = p.repeat;
    c.atomic_writers_per_addr = p.atomic_writers_per_addr;
    return c;
}
}  // namespace

CSR::CSR(const Defined::RowMajorMatrixXf& adj) {
    if (adj.rows() != adj.cols()) throw std::invalid_argument("Adjacency matrix must be square");
    int count = 0;
    for (long i = 0; i < adj.rows(); ++i) {
        RowOffset.push_back(count);
        for (long j = 0; j < adj.cols(); ++j) {
            if (adj(i, j) != 0) {
                ColInd.push_back(static_cast<int>(j));
                Value.push_back(adj(i, j));
                ++count;
            }
        }
    }
    RowOffset.push_back(count);
}

CSR_Order sortCSRByDegree(const CSR& csr, cwlb::Queue& q) {
    CSR_Order out;
    if (csr.RowOffset.size() < 2) return out;
    if (csr.ColInd.size() != csr.Value.size()) {
        throw std::runtime_error("CSR ColInd and Value size mismatch.");
    }
    const std::size_t rows = csr.RowOffset.size() - 1;
    if (rows > static_cast<std::size_t>(std::numeric_limits<int>::max()) ||
        csr.ColInd.size() > static_cast<std::size_t>(std::numeric_limits<int>::max())) {
        throw std::overflow_error(
            "DPL CPU degree reordering requires row and NNZ counts to fit in int.");
    }
    const int n = static_cast<int>(rows);
    const int nnz = static_cast<int>(csr.ColInd.size());
    out.Origin_local.resize(rows);
    out.RowOffset.resize(rows + 1);
    out.ColInd.resize(csr.ColInd.size());
    out.Value.resize(csr.Value.size());
    cwlb::check(cwlb_sort_by_degree(q.ctx(), n, nnz, csr.RowOffset.data(), csr.ColInd.data(),
                                    csr.Value.data(), out.Origin_local.data(), out.RowOffset.data(),
                                    out.ColInd.data(), out.Value.data()));
    return out;
}

CSR_Order sortCSRByDegree_SYCL(const CSR& csr, cwlb::Queue& q) { return sortCSRByDegree(csr, q); }

SpmmCostParams measure_spmm_costs(cwlb::Queue& q, int K, int repeat, int WI, int data_MB_for_load,
                                  int atomic_target_writers, const std::vector<int>&) {
    cwlb_costs c{};
    cwlb::check(cwlb_measure_spmm_costs(q.ctx(), K, repeat, WI, data_MB_for_load,
                                        atomic_target_writers, &c));
    SpmmCostParams p;
    p.C_compute_ns = c.C_compute_ns;
    p.C_load_ns = c.C_load_ns;
    p.C_store_ns = c.C_store_ns;
    p.C_atomic_ns = c.C_atomic_ns;
    p.K = c.K;
    p.WI = c.WI;
    p.repeat = c.repeat;
    p.atomic_writers_per_addr = c.atomic_writers_per_addr;
    return p;
}

std::vector<ParallelDataWeighted> costWeightedTaskPartitioning(cwlb::Queue& q,
                                                               const CSR_Order& csr,
                                                               const SpmmCostParams& costs,
                                                               double capacity_weight) {
    std::vector<ParallelDataWeighted> tasks;
    const int n = static_cast<int>(csr.RowOffset.size()) - 1;
    if (n <= 0) return tasks;
    const cwlb_costs c = to_c(costs);
    int64_t cnt = 0;
    // First call: the task count; second call: the task list.
    cwlb::check(cwlb_partition(q.ctx(), n, csr.RowOffset.data(), &c, capacity_weight, nullptr, 0, &cnt));
    tasks.resize(static_cast<std::size_t>(cnt));
    if (cnt > 0) {
        cwlb::check(cwlb_partition(q.ctx(), n, csr.RowOffset.data(), &c, capacity_weight,
                                   reinterpret_cast<cwlb_task*>(tasks.data()), cnt, &cnt));
    }
    return tasks;
}

std::vector<ParallelDataWeighted> costWeightedTaskPartitioning(const CSR_Order& csr,
                                                               const SpmmCostParams& costs,
                                                               double capacity_weight) {
    return costWeightedTaskPartitioning(cwlb::Queue::thread_default(), csr, costs, capacity_weight);
}

bool save_costs_one_per_line(SpmmCostParams costs, const std::string& filepath, bool append,
                             int precision) {
    const cwlb_costs c = to_c(costs);
    return cwlb_save_costs(&c, filepath.c_str(), append ? 1 : 0, precision) == CWLB_OK;
}

bool read_costs_one_per_line(SpmmCostParams& out, const std::string& filepath) {
    cwlb_costs c{};
    if (cwlb_read_costs(&c, filepath.c_str()) != CWLB_OK) return false;
    out.C_compute_ns = c.C_compute_ns;
    out.C_load_ns = c.C_load_ns;
    out.C_store_ns = c.C_store_ns;
    out.C_atomic_ns = c.C_atomic_ns;
    return true;
}

bool save_costs_per_k(const std::vector<SpmmCostParams>& table, const std::string& filepath) {
    std::vector<cwlb_costs> c;
    c.reserve(table.size());
    for (const SpmmCostParams& t : table) c.push_back(to_c(t));
    return cwlb_save_costs_per_k(c.data(), static_cast<int64_t>(c.size()), filepath.c_str()) ==
           CWLB_OK;
}

bool read_costs_per_k(std::vector<SpmmCostParams>& out, const std::string& filepath) {
    int64_t n = 0;
    if (cwlb_read_costs_per_k(nullptr, 0, filepath.c_str(), &n) != CWLB_OK) return false;
    std::vector<cwlb_costs> c(static_cast<size_t>(n));
    if (n > 0 && cwlb_read_costs_per_k(c.data(), n, filepath.c_str(), &n) != CWLB_OK) return false;
    out.clear();
    for (const cwlb_costs& e : c) {
        SpmmCostParams p;
        p.C_compute_ns = e.C_compute_ns;
        p.C_load_ns = e.C_load_ns;
        p.C_store_ns = e.C_store_ns;
        p.C_atomic_ns = e.C_atomic_ns;
        p.K = e.K;
        out.push_back(p);
    }
    return true;
}

SpmmCostParams costs_for_k(const std::vector<SpmmCostParams>& table, int K) {
    std::vector<cwlb_costs> c;
    c.reserve(table.size());
    for (const SpmmCostParams& t : table) c.push_back(to_c(t));
    const int64_t i = cwlb_costs_for_k(c.data(), static_cast<int64_t>(c.size()), K);
    if (i < 0) throw std::invalid_argument("no per-K cost entry for this K");
    return table[static_cast<size_t>(i)];
}

std::vector<std::pair<int, float>> get_csr_row_elements(const CSR& csr, int row) {
    std::vector<std::pair<int, float>> e;
    const int rows = static_cast<int>(csr.RowOffset.size()) - 1;
    if (row < 0 || row >= rows) return e;
    for (int i = csr.RowOffset[row]; i < csr.RowOffset[row + 1]; ++i) {
        e.emplace_back(csr.ColInd[i], csr.Value[i]);
    }
    return e;
}

bool validate_custom_csr_result(const Defined::RowMajorMatrixXf& result,
                                const Defined::RowMajorMatrixXf& reference, const CSR& csr,
                                const Defined::RowMajorMatrixXf& dense, float abs_tolerance) {
    int32_t passed = 0;
    cwlb::check(cwlb_validate_result(result.data(), result.rows(), result.cols(), reference.data(),
                                     reference.rows(), reference.cols(), csr.RowOffset.data(),
                                     static_cast<int64_t>(csr.RowOffset.size()),
                                     csr.ColInd.data(), csr.Value.data(), dense.data(),
                                     dense.rows(), dense.cols(), abs_tolerance, &passed));
    return passed != 0;
}

double capacity_from_s(int s, const SpmmCostParams& costs) {
    const cwlb_costs c = to_c(costs);
    return cwlb_capacity_from_s(s, &c);
}

int wave_based_s(const CSR_Order& sorted_csr, int compute_units, int wave) {
    if (compute_units <= 0 || wave <= 0) {
        throw std::invalid_argument("compute_units and wave must be positive.");
    }
    if (sorted_csr.RowOffset.empty()) return 1;
    int32_t s = 0;
    cwlb::check(cwlb_wave_based_s(static_cast<int64_t>(sorted_csr.RowOffset.back()), compute_units,
                                  wave, &s));
    return s;
}
