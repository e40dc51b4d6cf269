// CWLB-SpMM CPU oracle: a restatement of the reference's hot path.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and
// bench.py's CPU-baseline leg load this library, and only as the checker or
// as the timed CPU baseline; the product library (cwlb-spmm_b200/) never
// links, loads or calls it.
//
// Each function names the reference code it restates (paths are relative to
// the hhx-C/CWLB-SpMM project root).  Its behaviour is pinned by
// tests/test_oracle_pin.py against the reference's own sources compiled into
// oracle/_ref/libcwlbref.so, and by the golden fixtures in tests/golden/.
//
// Build: see oracle/Makefile (g++ -O3 -fopenmp -ffp-contract=off).  The
// double-precision partition arithmetic must not be contracted into FMAs:
// the reference's host code is compiled for baseline x86-64, which has none.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#include <omp.h>

namespace {

struct Task {
    int row_start;         // first reordered row, inclusive
    int row_end;           // last reordered row, exclusive
    int first_row_offset;  // nnz offset inside the first row
    int last_row_nnz;      // end offset inside the last row; 0 = full degree
};
static_assert(sizeof(Task) == 16, "ParallelDataWeighted is 4 x int32");

// x86-64 cvttsd2si semantics for double -> int32: values that do not fit
// (and NaN) produce INT32_MIN.  The reference relies on this implicitly in
// static_cast<int>(std::floor(...)) (src/utils.cpp:859-864).
int trunc_to_int_x86(double x) {
    if (x >= -2147483648.0 && x < 2147483648.0) return static_cast<int>(x);
    return INT32_MIN;
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Degree reordering, restating sortCSRByDegreeDPLCPU (main.cpp:197-278):
// rows ordered by (degree ascending, original id ascending); new offsets are
// the inclusive scan of the sorted degrees; rows copied unchanged.  A stable
// counting sort on degree yields exactly that order.
// Returns 0, or 2 when the result's nnz does not match (main.cpp:273-277).
int oracle_sort_by_degree(int n_rows, int nnz, const int* rowoff, const int* col,
                          const float* val, int* origin, int* new_rowoff, int* new_col,
                          float* new_val) {
    if (n_rows <= 0) return 0;
    int max_deg = 0;
    for (int r = 0; r < n_rows; ++r) max_deg = std::max(max_deg, rowoff[r + 1] - rowoff[r]);
    std::vector<int64_t> start(static_cast<size_t>(max_deg) + 2, 0);
    for (int r = 0; r < n_rows; ++r) start[rowoff[r + 1] - rowoff[r] + 1]++;
    for (size_t d = 1; d < start.size(); ++d) start[d] += start[d - 1];
    for (int r = 0; r < n_rows; ++r) origin[start[rowoff[r + 1] - rowoff[r]]++] = r;
    new_rowoff[0] = 0;
    for (int i = 0; i < n_rows; ++i) {
        const int o = origin[i];
        new_rowoff[i + 1] = new_rowoff[i] + (rowoff[o + 1] - rowoff[o]);
    }
#pragma omp parallel for schedule(dynamic, 1024)
    for (int i = 0; i < n_rows; ++i) {
        const int o = origin[i];
        const int len = rowoff[o + 1] - rowoff[o];
        std::memcpy(new_col + new_rowoff[i], col + rowoff[o], sizeof(int) * len);
        std::memcpy(new_val + new_rowoff[i], val + rowoff[o], sizeof(float) * len);
    }
    return new_rowoff[n_rows] == nnz ? 0 : 2;
}

// ---------------------------------------------------------------------------
// Cost-weighted task partitioning, restating costWeightedTaskPartitioning
// (src/utils.cpp:832-1021) step for step: complete rows are packed greedily
// under `capacity`; a row whose full weight exceeds it is cut into chunks of
// at most S nonzeros, the open task may absorb the row's (deg % S) prefix
// (:879-912), and a row's last chunk may absorb the next long row's prefix
// (:915-939).  costs = {C_compute, C_load, C_store, C_atomic}.
// `out` may be null (count only).  Returns the number of tasks.
int64_t oracle_partition(int n_rows, const int* rp, const double* costs, double capacity,
                         int* out, int64_t max_out) {
    if (n_rows <= 0) return 0;
    const double Cs = costs[2];
    const double Ca = costs[3];
    const double wCL = costs[0] + costs[1];
    const int S = std::max(1, trunc_to_int_x86(std::floor((capacity - Ca) / std::max(1e-30, wCL))));

    int64_t count = 0;
    int g_start = 0, first_off = 0, row = 0;
    double acc = 0.0;

    auto full_w = [&](int r) { return wCL * static_cast<double>(rp[r + 1] - rp[r]) + Cs; };
    auto chunk_w = [&](int nnz) { return wCL * static_cast<double>(nnz) + Ca; };
    auto emit = [&](int s, int e, int fo, int last) {
        if (s >= e) return;
        if (out && count < max_out) {
            out[4 * count + 0] = s;
            out[4 * count + 1] = e;
            out[4 * count + 2] = fo;
            out[4 * count + 3] = last;
        }
        ++count;
    };
    auto reset_at = [&](int r, int fo) {
        g_start = r;
        first_off = fo;
        acc = 0.0;
    };

    while (row < n_rows) {
        const int deg = rp[row + 1] - rp[row];
        const double wr = full_w(row);
        if (wr <= capacity) {
            if (acc == 0.0 || acc + wr <= capacity) {
                acc += wr;
                ++row;
            } else {
                emit(g_start, row, first_off, 0);
                reset_at(row, 0);
            }
            continue;
        }

        const bool absorbed = (acc == 0.0 && g_start == row && first_off > 0);
        int off = absorbed ? first_off : 0;
        int remaining = deg - off;
        if (remaining <= 0) {
            reset_at(row + 1, 0);
            ++row;
            continue;
        }
        if (!absorbed && !(acc <= 0.0)) {
            // Current task may take this row's (deg % S) prefix.
            const int r = deg % S;
            if (r == 0 || r >= deg) {
                emit(g_start, row, first_off, 0);
                reset_at(row, 0);
            } else if (chunk_w(r) <= capacity - acc) {
                emit(g_start, row + 1, first_off, r);
                reset_at(row, r);
                remaining -= r;
                off += r;
            } else {
                emit(g_start, row, first_off, 0);
                reset_at(row, 0);
            }
        }
        while (remaining > 0) {
            const int take = std::min(remaining, S);
            acc += chunk_w(take);
            remaining -= take;
            off += take;
            if (remaining > 0) {
                emit(g_start, row + 1, first_off, off);
                reset_at(row, off);
                continue;
            }
            // Last chunk: try to absorb the next long row's prefix.
            bool took_next = false;
            if (!(acc >= capacity) && row + 1 < n_rows) {
                const int nr = row + 1;
                const int nd = rp[nr + 1] - rp[nr];
                if (!(full_w(nr) <= capacity)) {
                    const int r2 = nd % S;
                    if (!(r2 == 0 || r2 >= nd)) {
                        const double w = chunk_w(r2);
                        const double rem = capacity - acc;
                        if (!(w > rem)) {
                            emit(g_start, nr + 1, first_off, r2);
                            reset_at(nr, r2);
                            took_next = true;
                        }
                    }
                }
            }
            if (!took_next) {
                emit(g_start, row + 1, first_off, 0);
                reset_at(row + 1, 0);
            }
        }
        ++row;
    }
    if (acc > 0.0 || g_start < n_rows) emit(g_start, n_rows, first_off, 0);
    return count;
}

// ---------------------------------------------------------------------------
// Mean aggregation, restating the semantics of spmmKernel and
// spmmKernelLargeKFallback (src/parallelMatrix.cpp:151-236, :411-664):
//   for every task, for every row r it covers, the fragment [begin, end) of
//   row r (begin = first_row_offset on the task's first row, end =
//   last_row_nnz on its last row when > 0, both clamped to [0, deg]) is
//   accumulated as acc = fma(value, H[col][k], acc) in nnz order, divided by
//   the row's full degree, and stored to out[origin[r]][k] when it is the
//   whole row or added to it otherwise.  Rows of degree 0 are left at 0.
// The reference merges fragments with unordered float atomics; this oracle
// adds them in task order, which is one of the orders the reference allows.
// H is h_rows x K row-major, out is n_rows x K row-major (original order).
// Returns 0, or 1 when an index is out of range.
int oracle_spmm_mean(int n_rows, const int* rowoff, const int* col, const float* val,
                     const int* origin, const float* H, int64_t h_rows, int64_t K,
                     const int* tasks, int64_t n_tasks, float* out, int n_threads) {
    if (n_threads > 0) omp_set_num_threads(n_threads);
    std::memset(out, 0, sizeof(float) * static_cast<size_t>(n_rows) * static_cast<size_t>(K));
    if (K == 0 || n_tasks == 0) return 0;
    for (int64_t t = 0; t < n_tasks; ++t) {
        const int* tk = tasks + 4 * t;
        if (tk[0] < 0 || tk[1] > n_rows) return 1;
    }
    for (int r = 0; r < n_rows; ++r) {
        if (origin[r] < 0 || origin[r] >= n_rows) return 1;
    }
    for (int j = 0; j < rowoff[n_rows]; ++j) {
        if (col[j] < 0 || col[j] >= h_rows) return 1;
    }

    struct Frag {
        int row, begin, end;
        int64_t task;
    };
    auto fragment = [&](const int* tk, int r, int& begin, int& end) -> bool {
        const int deg = rowoff[r + 1] - rowoff[r];
        if (deg <= 0) return false;
        begin = (r == tk[0]) ? tk[2] : 0;
        end = deg;
        if (r == tk[1] - 1 && tk[3] > 0) end = tk[3];
        begin = std::clamp(begin, 0, deg);
        end = std::clamp(end, begin, deg);
        return begin < end;
    };
    auto accumulate = [&](int r, int begin, int end, float* dst, bool add) {
        const int base = rowoff[r];
        const float deg = static_cast<float>(rowoff[r + 1] - base);
        for (int64_t k = 0; k < K; ++k) {
            float acc = 0.0f;
            for (int j = base + begin; j < base + end; ++j) {
                acc = std::fma(val[j], H[static_cast<int64_t>(col[j]) * K + k], acc);
            }
            acc /= deg;
            if (add) dst[k] += acc;
            else dst[k] = acc;
        }
    };

    // Whole rows: unique writers, any order.
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t t = 0; t < n_tasks; ++t) {
        const int* tk = tasks + 4 * t;
        for (int r = tk[0]; r < tk[1]; ++r) {
            int b, e;
            if (!fragment(tk, r, b, e)) continue;
            if (b == 0 && e == rowoff[r + 1] - rowoff[r]) {
                accumulate(r, b, e, out + static_cast<int64_t>(origin[r]) * K, false);
            }
        }
    }
    // Partial rows: only a task's first or last row can be partial.
    std::vector<Frag> frags;
    for (int64_t t = 0; t < n_tasks; ++t) {
        const int* tk = tasks + 4 * t;
        if (tk[0] >= tk[1]) continue;
        const int rows[2] = {tk[0], tk[1] - 1};
        for (int i = 0; i < (rows[0] == rows[1] ? 1 : 2); ++i) {
            int b, e;
            const int r = rows[i];
            if (!fragment(tk, r, b, e)) continue;
            if (b == 0 && e == rowoff[r + 1] - rowoff[r]) continue;
            frags.push_back({r, b, e, t});
        }
    }
    std::stable_sort(frags.begin(), frags.end(),
                     [](const Frag& a, const Frag& b) { return a.row < b.row; });
    std::vector<size_t> heads;
    for (size_t i = 0; i < frags.size(); ++i) {
        if (i == 0 || frags[i].row != frags[i - 1].row) heads.push_back(i);
    }
    heads.push_back(frags.size());
    const int64_t n_groups = static_cast<int64_t>(heads.size()) - 1;
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t h = 0; h < n_groups; ++h) {
        for (size_t i = heads[h]; i < heads[h + 1]; ++i) {
            const Frag& f = frags[i];
            accumulate(f.row, f.begin, f.end, out + static_cast<int64_t>(origin[f.row]) * K, true);
        }
    }
    return 0;
}

// Double-precision reference and error scale for the same aggregation,
// computed from the whole rows (every nonzero exactly once):
//   ref[o][k]  = (sum_j val_j * H[col_j][k]) / deg      (o = origin[r])
//   cond[o][k] = (sum_j |val_j * H[col_j][k]|) / deg
// Used by the parity tests: |gpu - ref| <= tol * max(|ref|, cond).
void oracle_spmm_mean_f64(int n_rows, const int* rowoff, const int* col, const float* val,
                          const int* origin, const float* H, int64_t K, double* ref,
                          double* cond, int n_threads) {
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 64)
    for (int r = 0; r < n_rows; ++r) {
        double* dst = ref + static_cast<int64_t>(origin[r]) * K;
        double* cdst = cond + static_cast<int64_t>(origin[r]) * K;
        const int deg = rowoff[r + 1] - rowoff[r];
        for (int64_t k = 0; k < K; ++k) {
            double s = 0.0, a = 0.0;
            for (int j = rowoff[r]; j < rowoff[r + 1]; ++j) {
                const double p = static_cast<double>(val[j]) *
                                 static_cast<double>(H[static_cast<int64_t>(col[j]) * K + k]);
                s += p;
                a += std::fabs(p);
            }
            dst[k] = deg > 0 ? s / deg : 0.0;
            cdst[k] = deg > 0 ? a / deg : 0.0;
        }
    }
}

// ---------------------------------------------------------------------------
// S-selection helpers, restating main.cpp.

// capacity_from_s (main.cpp:281-292)
double oracle_capacity_from_s(int s, const double* costs) {
    const double edge = costs[0] + costs[1];
    const int cs = std::max(1, s);
    if (edge <= 0.0) return std::max(0.0, costs[3]);
    return std::max(0.0, costs[3] + edge * static_cast<double>(cs));
}

// wave_based_s (main.cpp:295-321): S = max(1, ceil(nnz / (cu * w))), <= INT_MAX.
// Returns -1 for non-positive compute units or wave (std::invalid_argument).
int oracle_wave_based_s(int64_t nnz, int compute_units, int wave) {
    if (compute_units <= 0 || wave <= 0) return -1;
    const uint64_t n = static_cast<uint64_t>(nnz);
    const uint64_t d = static_cast<uint64_t>(compute_units) * static_cast<uint64_t>(wave);
    uint64_t s = (n + d - 1) / d;
    s = std::max<uint64_t>(1, s);
    s = std::min<uint64_t>(s, 2147483647ULL);
    return static_cast<int>(s);
}

// recommended_candidate_w (main.cpp:87-95): the w table keyed by nnz.
void oracle_recommended_w(uint64_t nnz, int* out) {
    static const uint64_t limit[6] = {100000ULL, 500000ULL, 1000000ULL,
                                      5000000ULL, 10000000ULL, 50000000ULL};
    static const int first[7] = {64, 128, 256, 512, 1024, 4096, 8192};
    int i = 0;
    while (i < 6 && nnz >= limit[i]) ++i;
    out[0] = first[i];
    out[1] = first[i] / 2;
    out[2] = first[i] / 4;
}

// deterministic_features (main.cpp:324-336): mt19937(42), U[0,1) floats,
// row-major.  Uses the same libstdc++ engine and distribution.
void oracle_features(int rows, int cols, float* out) {
    std::mt19937 gen(42);
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    const int64_t n = static_cast<int64_t>(rows) * cols;
    for (int64_t i = 0; i < n; ++i) out[i] = dist(gen);
}

}  // extern "C"
