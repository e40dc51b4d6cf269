#pragma once
// Text CSR loading (reference: include/data.h:8, src/data.cpp:12-130).
#include <string>

#include "Matrix.h"

// Loads "<dataset dir><name>[.csr]": line 1 = row offsets, line 2 = column
// ids, comma separated; all values are 1.0f.  V = rows, E = nnz.  Throws
// std::runtime_error with the reference's messages on malformed input, and
// std::invalid_argument / std::out_of_range for cells that are not integers
// (as std::stoi does).
CSR loadDatasetToCSR(const std::string& datasetName, int& V, int& E);

// The same parser on an explicit file path.
CSR loadTextCSRPath(const std::string& path, int& V, int& E);
