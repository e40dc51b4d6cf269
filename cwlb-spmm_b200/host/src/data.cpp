// Text CSR loader (reference: src/data.cpp:12-130).
//
// File format: line 1 = row offsets, line 2 = column ids, comma separated.
// The reference reads both lines with std::getline and converts every
// non-empty comma-separated cell with std::stoi; this loader reads the file
// in one block and parses in place, with the same acceptance rules
// (std::stoi skips leading white space, takes an optional sign and the
// following digits, ignores what trails them, throws std::invalid_argument
// without digits and std::out_of_range outside int) and the same checks and
// messages, in the same order.
#include <cctype>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "data.h"

namespace {

bool ends_with(const std::string& s, const std::string& suffix) {
    return s.size() >= suffix.size() &&
           s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0;
}

int parse_cell(const char* p, const char* e) {
    while (p < e && std::isspace(static_cast<unsigned char>(*p))) ++p;
    bool neg = false;
    if (p < e && (*p == '+' || *p == '-')) {
        neg = *p == '-';
        ++p;
    }
    if (p >= e || !std::isdigit(static_cast<unsigned char>(*p))) throw std::invalid_argument("stoi");
    int64_t v = 0;
    bool overflow = false;
    for (; p < e && std::isdigit(static_cast<unsigned char>(*p)); ++p) {
        if (!overflow) {
            v = v * 10 + (*p - '0');
            if (v > 2147483648LL) overflow = true;
        }
    }
    if (neg) v = -v;
    if (overflow || v > 2147483647LL || v < -2147483648LL) throw std::out_of_range("stoi");
    return static_cast<int>(v);
}

void parse_line(const char* b, const char* e, std::vector<int>& out) {
    const char* cell = b;
    for (const char* p = b;; ++p) {
        if (p == e || *p == ',') {
            if (p > cell) out.push_back(parse_cell(cell, p));
            if (p == e) break;
            cell = p + 1;
        }
    }
}

}  // namespace

CSR loadTextCSRPath(const std::string& path, int& V, int& E) {
    CSR csr;
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("Failed to open .csr file: " + path);
    std::string buf;
    {
        char chunk[1 << 16];
        size_t n;
        while ((n = std::fread(chunk, 1, sizeof(chunk), f)) > 0) buf.append(chunk, n);
        std::fclose(f);
    }
    const char* b = buf.data();
    const char* end = b + buf.size();
    if (buf.empty()) throw std::runtime_error("Failed to read the first line of .csr file: " + path);
    const char* nl1 = b;
    while (nl1 < end && *nl1 != '\n') ++nl1;
    parse_line(b, nl1, csr.RowOffset);
    if (nl1 >= end || nl1 + 1 >= end) {
        throw std::runtime_error("Failed to read the second line of .csr file: " + path);
    }
    const char* b2 = nl1 + 1;
    const char* nl2 = b2;
    while (nl2 < end && *nl2 != '\n') ++nl2;
    parse_line(b2, nl2, csr.ColInd);

    if (csr.RowOffset.empty()) throw std::runtime_error(".csr file has an empty RowOffset: " + path);
    V = static_cast<int>(csr.RowOffset.size()) - 1;
    E = csr.RowOffset.back();
    if (V < 0) throw std::runtime_error("Invalid RowOffset size. It should be vertex_count + 1");
    if (E < 0) throw std::runtime_error("RowOffset.back(), namely NNZ, is negative");
    if (static_cast<int64_t>(csr.ColInd.size()) != E) {
        throw std::runtime_error("ColInd size does not match RowOffset.back()(NNZ): ColInd=" +
                                 std::to_string(csr.ColInd.size()) + ", NNZ=" + std::to_string(E));
    }
    if (csr.RowOffset.front() != 0) {
        throw std::runtime_error("RowOffset[0] must be 0, current value is " +
                                 std::to_string(csr.RowOffset.front()));
    }
    for (std::size_t i = 1; i < csr.RowOffset.size(); ++i) {
        if (csr.RowOffset[i] < csr.RowOffset[i - 1]) {
            throw std::runtime_error("RowOffset is not monotonically non-decreasing at index " +
                                     std::to_string(i));
        }
        if (csr.RowOffset[i] > E) {
            throw std::runtime_error("RowOffset contains a value larger than NNZ at index " +
                                     std::to_string(i));
        }
    }
    for (int c : csr.ColInd) {
        if (c < 0) throw std::runtime_error("ColInd contains a negative column index");
    }
    csr.Value.assign(csr.ColInd.size(), 1.0f);
    return csr;
}

CSR loadDatasetToCSR(const std::string& datasetName, int& V, int& E) {
    if (datasetName.empty()) throw std::runtime_error("Dataset name is empty");
    const std::string name = ends_with(datasetName, ".csr") ? datasetName : datasetName + ".csr";
    const char* dir = std::getenv("CWLB_DATASET_DIR");
    std::string base = dir ? std::string(dir) : std::string(DATA_CSR_FILE_PATH);
    if (dir && !base.empty() && base.back() != '/') base += '/';
    return loadTextCSRPath(base + name, V, E);
}
