#pragma once
// Task and cost structures and helper functions of the CWLB-SpMM interface
// (reference: include/utils.h:13-83).  The sort, the partitioner and the
// calibration run on the B200 through libcwlb_spmm.
#include <string>
#include <utility>
#include <vector>

#include "Matrix.h"
#include "config.h"
#include "cwlb_queue.h"

struct ParallelDataWeighted {
    int row_start;         // first reordered row, inclusive
    int row_end;           // last reordered row, exclusive
    int first_row_offset;  // nonzero offset within the first row
    int last_row_nnz;      // end offset within the last row; 0 = full degree
};

// Calibrated relative weights (ns x 10 per operation) and calibration metadata.
struct SpmmCostParams {
    double C_compute_ns = 0.0;
    double C_load_ns = 0.0;
    double C_store_ns = 0.0;
    double C_atomic_ns = 0.0;
    int K = 0;
    int WI = 0;
    int repeat = 0;
    int atomic_writers_per_addr = 0;
};

// Details of one failed element of validate_custom_csr_result.
struct ErrorElement {
    int result_row = 0;
    int result_col = 0;
    float sycl_value = 0.0f;
    float reference_value = 0.0f;
    float absolute_error = 0.0f;
    std::vector<std::pair<int, float>> csr_row_elements;
    std::vector<float> dense_col_elements;
};

// Rows ordered by (degree, original id), offsets rescanned, rows copied:
// the reference's sortCSRByDegreeDPLCPU (main.cpp:197-278), on the GPU.
CSR_Order sortCSRByDegree(const CSR& csr, cwlb::Queue& q);

// sortCSRByDegree_SYCL (include/utils.h:13, src/utils.cpp:104-339): the
// reference's optional GPU bucket ordering, whose ties come out in any order.
// Here the same device sort as above: ascending degree, ties by original id
// (one of the orders the bucket sort may produce).
CSR_Order sortCSRByDegree_SYCL(const CSR& csr, cwlb::Queue& q);

// measure_spmm_costs (utils.h:47-54): the four calibration microbenchmarks.
SpmmCostParams measure_spmm_costs(cwlb::Queue& q, int K = 128, int repeat = 500,
                                  int WI = 131072, int data_MB_for_load = 512,
                                  int atomic_target_writers = 8,
                                  const std::vector<int>& atomic_group_candidates = {});

// costWeightedTaskPartitioning (utils.h:57-60) on the GPU; the queue-less
// form uses the calling thread's default queue.
std::vector<ParallelDataWeighted> costWeightedTaskPartitioning(const CSR_Order& csr,
                                                               const SpmmCostParams& costs,
                                                               double capacity_weight);
std::vector<ParallelDataWeighted> costWeightedTaskPartitioning(cwlb::Queue& q,
                                                               const CSR_Order& csr,
                                                               const SpmmCostParams& costs,
                                                               double capacity_weight);

// Cost file: compute, load, store, atomic; one coefficient per line.
bool save_costs_one_per_line(SpmmCostParams costs, const std::string& filepath = COSTFILEPATH,
                             bool append = false, int precision = 6);
bool read_costs_one_per_line(SpmmCostParams& out, const std::string& filepath = COSTFILEPATH);

// Per-K cost table, an extension of the cost file (cwlb_save_costs_per_k):
// one "K C_compute C_load C_store C_atomic" line per calibrated row width K.
bool save_costs_per_k(const std::vector<SpmmCostParams>& table,
                      const std::string& filepath = COSTFILEPATH_PER_K);
bool read_costs_per_k(std::vector<SpmmCostParams>& out,
                      const std::string& filepath = COSTFILEPATH_PER_K);
// The entry calibrated at the row width nearest to K on a log scale (ties go
// to the larger width); std::invalid_argument for an empty table or K <= 0.
SpmmCostParams costs_for_k(const std::vector<SpmmCostParams>& table, int K);

std::vector<std::pair<int, float>> get_csr_row_elements(const CSR& csr, int row);

// Compares a result against a caller-supplied reference with an absolute
// tolerance (NaN/Inf aware); prints up to 10 mismatches.
bool validate_custom_csr_result(const Defined::RowMajorMatrixXf& result,
                                const Defined::RowMajorMatrixXf& reference, const CSR& csr,
                                const Defined::RowMajorMatrixXf& dense_matrix,
                                float abs_tolerance = 1e-4f);

// S-selection helpers of the reference's main.cpp (:87-95, :281-321).
double capacity_from_s(int s, const SpmmCostParams& costs);
int wave_based_s(const CSR_Order& sorted_csr, int compute_units, int wave);
