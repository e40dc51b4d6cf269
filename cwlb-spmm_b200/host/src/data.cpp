// Text CSR loader (reference: src/data.cpp:12-130).
//
// File format: line 1 = row offsets, line 2 = column ids, comma separated.
// The reference reads both lines with std::getline and converts every
// non-empty comma-separated cell with std::stoi; this loader reads the file
// in one block and parses in place, with the same acceptance rules
// (std::stoi skips leading white space, takes an optional sign and the
// following digits, ignores what trails them, throws std::invalid_argument
// without digits and std::out_of_range outside int) and the same checks and
// messages, in the same order.  Lines of 8 MB and more are parsed by up to 16
// threads, in pieces cut at commas; the first bad cell in line order decides
// the error, as in a sequential parse.
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <thread>
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

// parse_line over up to 16 host threads for long lines: the line is cut at
// commas into contiguous pieces, each piece parsed on its own, the values
// concatenated in order.  If several pieces hold a bad cell, the error of the
// earliest piece is the one raised, as a sequential parse would raise it.
void parse_line_parallel(const char* b, const char* e, std::vector<int>& out) {
    const size_t len = static_cast<size_t>(e - b);
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const unsigned T = static_cast<unsigned>(std::min<size_t>(std::min(16u, hw), len >> 22));
    if (T <= 1) {
        parse_line(b, e, out);
        return;
    }
    std::vector<const char*> cut(T + 1);
    cut[0] = b;
    cut[T] = e;
    for (unsigned t = 1; t < T; ++t) {
        const char* p = std::max(cut[t - 1], b + len / T * t);
        while (p < e && *p != ',') ++p;  // a piece starts at a comma: its first cell is empty
        cut[t] = p;
    }
    std::vector<std::vector<int>> part(T);
    std::vector<std::exception_ptr> err(T);
    auto work = [&](unsigned t) {
        try {
            parse_line(cut[t], cut[t + 1], part[t]);
        } catch (...) {
            err[t] = std::current_exception();
        }
    };
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < T; ++t) pool.emplace_back(work, t);
    work(0);
    for (auto& th : pool) th.join();
    for (unsigned t = 0; t < T; ++t)
        if (err[t]) std::rethrow_exception(err[t]);
    size_t total = out.size();
    for (const auto& v : part) total += v.size();
    out.reserve(total);
    for (const auto& v : part) out.insert(out.end(), v.begin(), v.end());
}

}  // namespace

CSR loadTextCSRPath(const std::string& path, int& V, int& E) {
    CSR csr;
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("Failed to open .csr file: " + path);
    std::string buf;
    {
        // One read of the whole file when its size is known, then whatever
        // follows (a file that grew, or a stream without a size).
        struct stat st {};
        size_t got = 0;
        if (::fstat(::fileno(f), &st) == 0 && st.st_size > 0) {
            buf.resize(static_cast<size_t>(st.st_size));
            got = std::fread(&buf[0], 1, buf.size(), f);
            buf.resize(got);
        }
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
    parse_line_parallel(b, nl1, csr.RowOffset);
    if (nl1 >= end || nl1 + 1 >= end) {
        throw std::runtime_error("Failed to read the second line of .csr file: " + path);
    }
    const char* b2 = nl1 + 1;
    const char* nl2 = b2;
    while (nl2 < end && *nl2 != '\n') ++nl2;
    parse_line_parallel(b2, nl2, csr.ColInd);

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

namespace {

std::string dataset_path(const std::string& datasetName) {
    if (datasetName.empty()) throw std::runtime_error("Dataset name is empty");
    const std::string name = ends_with(datasetName, ".csr") ? datasetName : datasetName + ".csr";
    const char* dir = std::getenv("CWLB_DATASET_DIR");
    std::string base = dir ? std::string(dir) : std::string(DATA_CSR_FILE_PATH);
    if (dir && !base.empty() && base.back() != '/') base += '/';
    return base + name;
}

}  // namespace

CSR loadDatasetToCSR(const std::string& datasetName, int& V, int& E) {
    return loadTextCSRPath(dataset_path(datasetName), V, E);
}

// ---------------------------------------------------------------------------
// Binary cache.

namespace {

constexpr char kCacheMagic[8] = {'C', 'W', 'L', 'B', 'C', 'S', 'R', '1'};
constexpr uint32_t kCacheVersion = 1;

struct CacheHeader {
    char magic[8];
    uint32_t version;
    uint32_t header_bytes;
    uint64_t source_size;
    int64_t source_mtime_ns;
    int64_t rows;
    int64_t nnz;
    uint64_t checksum;
    uint64_t reserved;
};
static_assert(sizeof(CacheHeader) == 64, "cache header layout");

bool source_stamp(const std::string& path, uint64_t& size, int64_t& mtime_ns) {
    struct stat st {};
    if (::stat(path.c_str(), &st) != 0) return false;
    size = static_cast<uint64_t>(st.st_size);
    mtime_ns = static_cast<int64_t>(st.st_mtim.tv_sec) * 1000000000LL + st.st_mtim.tv_nsec;
    return true;
}

// FNV-1a over 32-bit words.
uint64_t checksum_words(const int* p, std::size_t n, uint64_t h) {
    for (std::size_t i = 0; i < n; ++i) {
        h ^= static_cast<uint32_t>(p[i]);
        h *= 1099511628211ULL;
    }
    return h;
}

uint64_t csr_checksum(const CSR& csr) {
    const uint64_t h = checksum_words(csr.RowOffset.data(), csr.RowOffset.size(),
                                      1469598103934665603ULL);
    return checksum_words(csr.ColInd.data(), csr.ColInd.size(), h);
}

}  // namespace

std::string csrCachePath(const std::string& text_path) { return text_path + ".cwlbbin"; }

bool writeCSRCache(const CSR& csr, const std::string& text_path) {
    CacheHeader h{};
    std::memcpy(h.magic, kCacheMagic, sizeof(h.magic));
    h.version = kCacheVersion;
    h.header_bytes = sizeof(CacheHeader);
    if (!source_stamp(text_path, h.source_size, h.source_mtime_ns)) return false;
    if (csr.RowOffset.empty()) return false;
    h.rows = static_cast<int64_t>(csr.RowOffset.size()) - 1;
    h.nnz = static_cast<int64_t>(csr.ColInd.size());
    h.checksum = csr_checksum(csr);
    const std::string final_path = csrCachePath(text_path);
    const std::string tmp = final_path + ".tmp" + std::to_string(static_cast<long>(::getpid()));
    std::FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) return false;
    bool ok = std::fwrite(&h, sizeof(h), 1, f) == 1 &&
              std::fwrite(csr.RowOffset.data(), sizeof(int), csr.RowOffset.size(), f) ==
                  csr.RowOffset.size() &&
              (csr.ColInd.empty() ||
               std::fwrite(csr.ColInd.data(), sizeof(int), csr.ColInd.size(), f) ==
                   csr.ColInd.size());
    ok = (std::fclose(f) == 0) && ok;
    if (ok) ok = std::rename(tmp.c_str(), final_path.c_str()) == 0;
    if (!ok) std::remove(tmp.c_str());
    return ok;
}

bool readCSRCache(const std::string& text_path, CSR& csr, int& V, int& E) {
    uint64_t size = 0;
    int64_t mtime = 0;
    if (!source_stamp(text_path, size, mtime)) return false;
    std::FILE* f = std::fopen(csrCachePath(text_path).c_str(), "rb");
    if (!f) return false;
    CacheHeader h{};
    CSR c;
    bool ok = std::fread(&h, sizeof(h), 1, f) == 1 &&
              std::memcmp(h.magic, kCacheMagic, sizeof(h.magic)) == 0 &&
              h.version == kCacheVersion && h.header_bytes == sizeof(CacheHeader) &&
              h.source_size == size && h.source_mtime_ns == mtime && h.rows >= 0 &&
              h.rows < INT_MAX && h.nnz >= 0 && h.nnz <= INT_MAX;
    if (ok) {
        // The file must hold exactly the two arrays after the header.
        const long want = static_cast<long>(sizeof(CacheHeader)) + 4L * (h.rows + 1) + 4L * h.nnz;
        ok = std::fseek(f, 0, SEEK_END) == 0 && std::ftell(f) == want &&
             std::fseek(f, static_cast<long>(sizeof(CacheHeader)), SEEK_SET) == 0;
    }
    if (ok) {
        c.RowOffset.resize(static_cast<std::size_t>(h.rows) + 1);
        c.ColInd.resize(static_cast<std::size_t>(h.nnz));
        ok = std::fread(c.RowOffset.data(), sizeof(int), c.RowOffset.size(), f) ==
                 c.RowOffset.size() &&
             (c.ColInd.empty() ||
              std::fread(c.ColInd.data(), sizeof(int), c.ColInd.size(), f) == c.ColInd.size());
    }
    std::fclose(f);
    if (!ok || csr_checksum(c) != h.checksum || c.RowOffset.front() != 0 ||
        c.RowOffset.back() != h.nnz) {
        return false;
    }
    // The invariants the text loader checked before the cache was written.
    for (std::size_t i = 1; i < c.RowOffset.size(); ++i) {
        if (c.RowOffset[i] < c.RowOffset[i - 1]) return false;
    }
    for (int col : c.ColInd) {
        if (col < 0) return false;
    }
    c.Value.assign(c.ColInd.size(), 1.0f);
    V = static_cast<int>(h.rows);
    E = static_cast<int>(h.nnz);
    csr = std::move(c);
    return true;
}

CSR loadTextCSRPathCached(const std::string& path, int& V, int& E, CsrCacheStatus* status) {
    CSR csr;
    if (readCSRCache(path, csr, V, E)) {
        if (status) *status = CsrCacheStatus::Hit;
        return csr;
    }
    csr = loadTextCSRPath(path, V, E);
    const bool written = writeCSRCache(csr, path);
    if (status) *status = written ? CsrCacheStatus::Written : CsrCacheStatus::NotWritten;
    return csr;
}

CSR loadDatasetToCSRCached(const std::string& datasetName, int& V, int& E,
                           CsrCacheStatus* status) {
    return loadTextCSRPathCached(dataset_path(datasetName), V, E, status);
}
