#pragma once
// Timing settings, run-time paths and the dense-matrix type of the CWLB-SpMM
// C++ interface (reference: include/config.h:1-25), for the B200 build.
//
// The paths keep the reference's defaults (relative to a build/ working
// directory); the dataset loader honours CWLB_DATASET_DIR, and the cwlb-spmm
// and costWrite tools CWLB_COSTFILE, CWLB_COSTFILE_PER_K and CWLB_RESULTS.
#include <cstddef>
#include <stdexcept>
#include <string>
#include <vector>

// As in the reference's config.h: code written against it may rely on this.
using namespace std;

// Timed samples = LOOPCOUNT - WARMUPCOUNT; LOOPCOUNT includes the warm-up.
inline const int WARMUPCOUNT = 20;
inline const int LOOPCOUNT = 70;
inline const std::string COSTFILEPATH = "../resources/spmm_costs.txt";
// Per-K cost table (costWrite --per-k; an extension of the cost file).
inline const std::string COSTFILEPATH_PER_K = "../resources/spmm_costs_per_k.txt";
constexpr const char* DATA_CSR_FILE_PATH = "../resources/datasets/";

namespace Defined {

// Dense row-major float matrix: adjacent feature columns are contiguous.  It
// provides what the interface uses from the reference's Eigen row-major matrix:
// rows(), cols(), data(), element access and Zero().
class RowMajorMatrixXf {
public:
    RowMajorMatrixXf() = default;
    RowMajorMatrixXf(long rows, long cols) : rows_(rows), cols_(cols) {
        if (rows < 0 || cols < 0) throw std::invalid_argument("negative matrix size");
        v_.assign(static_cast<std::size_t>(rows) * static_cast<std::size_t>(cols), 0.0f);
    }
    static RowMajorMatrixXf Zero(long rows, long cols) { return RowMajorMatrixXf(rows, cols); }
    long rows() const { return rows_; }
    long cols() const { return cols_; }
    float* data() { return v_.data(); }
    const float* data() const { return v_.data(); }
    float& operator()(long i, long j) { return v_[static_cast<std::size_t>(i * cols_ + j)]; }
    float operator()(long i, long j) const { return v_[static_cast<std::size_t>(i * cols_ + j)]; }

private:
    long rows_ = 0;
    long cols_ = 0;
    std::vector<float> v_;
};

}  // namespace Defined
