// cwlb_validate_result: the reference's result check, validate_custom_csr_result
// (src/utils.cpp:1095-1265), on host arrays.  Host code only; the C++
// interface's validate_custom_csr_result (host/src/utils.cpp) calls it.
//
// The report format is the interface: a pass line, or up to 10 mismatches,
// each with the CSR row's stored entries, the first 5 entries of the dense
// matrix's column and the two values.  Stream formatting is not reset, as in
// the reference: the fixed/6-digit mode set for the first printed value stays
// in effect on std::cout afterwards.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <iomanip>
#include <iostream>
#include <limits>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "cwlb_spmm.h"

namespace cwlb {
void set_last_error(const std::string& msg);
}

namespace {

struct Mismatch {
    int64_t row = 0, col = 0;
    float got = 0.0f, want = 0.0f, abs_err = 0.0f;
    std::vector<std::pair<int32_t, float>> row_entries;
    std::vector<float> dense_col;
};

// The report below (get_csr_row_elements and validate_custom_csr_result,
// src/utils.cpp:1095-1265 of hhx-C/CWLB-SpMM) restates the reference's
// checks, their order and its output text, which callers compare byte for
// byte.  That code is Copyright (c) 2026, Hongxing He, Guanlin He and Chunlin
// Li, under the BSD 3-Clause License: redistribution and use in source and
// binary forms, with or without modification, are permitted provided that
// the copyright notice, this list of conditions and the disclaimer are
// retained; neither the names of the copyright holders nor of the
// contributors may be used to endorse or promote derived products without
// prior written permission.  THE SOFTWARE IS PROVIDED "AS IS", WITHOUT
// WARRANTY OF ANY KIND.

// get_csr_row_elements (src/utils.cpp:1095-1115): empty outside [0, rows).
std::vector<std::pair<int32_t, float>> row_entries(const int32_t* row_offset, int64_t len,
                                                   const int32_t* col, const float* val,
                                                   int64_t row) {
    std::vector<std::pair<int32_t, float>> e;
    if (row < 0 || row >= len - 1) return e;
    for (int32_t i = row_offset[row]; i < row_offset[row + 1]; ++i) e.emplace_back(col[i], val[i]);
    return e;
}

bool compare(const float* result, int64_t rr, int64_t rc, const float* ref, int64_t fr, int64_t fc,
             const int32_t* row_offset, int64_t ro_len, const int32_t* col, const float* val,
             const float* dense, int64_t dr, int64_t dc, float tol) {
    try {
        if (tol < 0.0f || !std::isfinite(tol)) {
            throw std::invalid_argument("Validation tolerance must be finite and non-negative.");
        }
        if (rr != fr || rc != fc) {
            std::cerr << "Validation failed: result matrix shape is (" << rr << ", " << rc
                      << "), but reference matrix shape is (" << fr << ", " << fc << ").\n";
            return false;
        }
        if (ro_len != fr + 1) {
            std::cerr << "Validation failed: CSR row count does not match the reference matrix.\n";
            return false;
        }
        if (dr <= 0 || dc != fc) {
            std::cerr << "Validation failed: input dense matrix shape is incompatible with the "
                         "reference result.\n";
            return false;
        }
        std::vector<Mismatch> bad;
        for (int64_t r = 0; r < fr && bad.size() < 10; ++r) {
            for (int64_t c = 0; c < fc && bad.size() < 10; ++c) {
                const float got = result[r * rc + c];
                const float want = ref[r * fc + c];
                bool mismatch;
                float err;
                if (std::isnan(got) || std::isnan(want)) {
                    mismatch = !(std::isnan(got) && std::isnan(want));
                    err = mismatch ? std::numeric_limits<float>::infinity() : 0.0f;
                } else if (std::isinf(got) || std::isinf(want)) {
                    mismatch = got != want;
                    err = mismatch ? std::numeric_limits<float>::infinity() : 0.0f;
                } else {
                    err = std::abs(got - want);
                    mismatch = err > tol;
                }
                if (!mismatch) continue;
                Mismatch m;
                m.row = r;
                m.col = c;
                m.got = got;
                m.want = want;
                m.abs_err = err;
                m.row_entries = row_entries(row_offset, ro_len, col, val, r);
                m.dense_col.resize(static_cast<std::size_t>(dr));
                for (int64_t d = 0; d < dr; ++d) m.dense_col[d] = dense[d * dc + c];
                bad.push_back(std::move(m));
            }
        }
        if (bad.empty()) {
            std::cout << "\033[1;32mValidation passed: all elements satisfy the comparison "
                         "criteria.\033[0m\n";
            return true;
        }
        std::cout << "\033[1;31mValidation failed: showing " << bad.size()
                  << " mismatched elements (up to the first 10).\033[0m\n";
        for (std::size_t i = 0; i < bad.size(); ++i) {
            const Mismatch& m = bad[i];
            std::cout << "\nStored entries in CSR row " << m.row << ":\n";
            std::cout << "RowOffset[" << m.row << "]: " << row_offset[m.row] << '\n';
            std::cout << "RowOffset[" << m.row + 1 << "]: " << row_offset[m.row + 1] << '\n';
            std::cout << "Format: [ColInd] -> Value\n";
            for (const auto& e : m.row_entries) {
                std::cout << "  [" << e.first << "] -> " << e.second << '\n';
            }
            std::cout << "\nDense matrix column " << m.col << " (up to the first 5 rows):\n";
            const int shown = static_cast<int>(std::min<std::size_t>(5, m.dense_col.size()));
            for (int d = 0; d < shown; ++d) std::cout << "  Row " << d << ": " << m.dense_col[d] << '\n';
            std::cout << "\n\033[1;34mMismatch #" << i + 1 << ":\033[0m\n";
            std::cout << "Result matrix position: (" << m.row << ", " << m.col << ")\n";
            std::cout << std::fixed << std::setprecision(6);
            std::cout << "SYCL result:     " << m.got << '\n';
            std::cout << "Reference value: " << m.want << '\n';
            std::cout << "Absolute error:  " << m.abs_err << '\n';
        }
        return false;
    } catch (const std::exception& e) {
        std::cerr << "Validation error: " << e.what() << '\n';
        return false;
    }
}

}  // namespace

extern "C" int cwlb_validate_result(const float* result, int64_t result_rows, int64_t result_cols,
                                    const float* reference, int64_t reference_rows,
                                    int64_t reference_cols, const int32_t* row_offset,
                                    int64_t row_offset_len, const int32_t* col_ind,
                                    const float* value, const float* dense, int64_t dense_rows,
                                    int64_t dense_cols, float abs_tolerance, int32_t* passed) {
    if (!passed || result_rows < 0 || result_cols < 0 || reference_rows < 0 ||
        reference_cols < 0 || row_offset_len < 0 || dense_rows < 0 || dense_cols < 0) {
        cwlb::set_last_error("cwlb_validate_result: null output or negative size");
        return CWLB_ERR_INVALID_ARGUMENT;
    }
    *passed = compare(result, result_rows, result_cols, reference, reference_rows, reference_cols,
                      row_offset, row_offset_len, col_ind, value, dense, dense_rows, dense_cols,
                      abs_tolerance)
                  ? 1
                  : 0;
    return CWLB_OK;
}
