#pragma once
// CSR storage of the CWLB-SpMM interface (reference: include/Matrix.h:15-36).
// The standard headers the reference's Matrix.h brings in are included too,
// since code written against it may use them through this header.
#include <fstream>
#include <iostream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "config.h"

// Standard CSR: row offsets index the column/value arrays.
class CSR {
public:
    std::vector<int> RowOffset;
    std::vector<int> ColInd;
    std::vector<float> Value;

    // Dense (square) adjacency matrix to CSR, keeping the non-zero entries
    // row by row (reference: src/Matrix.cpp:14-52).
    explicit CSR(const Defined::RowMajorMatrixXf& adj);
    CSR(std::vector<int> row_offset, std::vector<int> col_ind, std::vector<float> value)
        : RowOffset(std::move(row_offset)), ColInd(std::move(col_ind)), Value(std::move(value)) {}
    CSR() = default;
};

// Degree-reordered CSR with the row mapping used to restore output order.
class CSR_Order {
public:
    std::vector<int> Origin_local;  // reordered row -> original row id
    std::vector<int> RowOffset;
    std::vector<int> ColInd;
    std::vector<float> Value;
};
