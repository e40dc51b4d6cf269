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

// ------------------------------------------------------------------------
// Binary cache beside a text CSR (no counterpart in the reference, whose
// loader parses the text on every run).  "<file>.csr.cwlbbin" holds a 64-byte
// header (magic "CWLBCSR1", version 1, the text file's size and modification
// time in ns, V, E, a 64-bit checksum of the arrays) and then RowOffset
// (int32[V+1]) and ColInd (int32[E]); values are all 1.0f, as the text
// loader makes them.  A cache whose source size or time differs from the
// text file's, or whose size or checksum is wrong, is ignored.

enum class CsrCacheStatus { Hit, Written, NotWritten };

// Path of the cache that belongs to a text file.
std::string csrCachePath(const std::string& text_path);

// Writes the cache of `csr` (as loaded from text_path).  Written to a
// temporary file and renamed, so readers never see a partial cache.
// Returns false (and leaves no file) on any failure.
bool writeCSRCache(const CSR& csr, const std::string& text_path);

// Reads the cache of text_path; false if it is missing, stale or corrupt.
bool readCSRCache(const std::string& text_path, CSR& csr, int& V, int& E);

// loadTextCSRPath through the cache: a fresh cache is read; otherwise the
// text is parsed (same checks and errors as loadTextCSRPath) and the cache
// written.  `status`, if given, says which happened.
CSR loadTextCSRPathCached(const std::string& path, int& V, int& E,
                          CsrCacheStatus* status = nullptr);

// loadDatasetToCSR through the cache.
CSR loadDatasetToCSRCached(const std::string& datasetName, int& V, int& E,
                           CsrCacheStatus* status = nullptr);
