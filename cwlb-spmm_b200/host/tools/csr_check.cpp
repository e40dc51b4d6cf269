// csr-check: loads a text .csr file with the cwlb-spmm loader and prints
// "V E checksum" (checksum = FNV-1a over the offsets and column ids), or the
// loader's error message on stderr with exit status 1.  Useful to validate a
// dataset before a long run.  With --cache the file is loaded through the
// binary cache beside it (read when fresh, written otherwise), and stderr
// says which: "cache: hit", "cache: written" or "cache: not written".
//   csr-check [--cache] <path-to-file.csr>
#include <cstdint>
#include <cstdio>
#include <iostream>
#include <stdexcept>
#include <string>

#include "data.h"

int main(int argc, char** argv) {
    const bool cache = argc == 3 && std::string(argv[1]) == "--cache";
    if (argc != 2 && !cache) {
        std::cerr << "Usage: csr-check [--cache] <file.csr>\n";
        return 1;
    }
    try {
        int V = 0, E = 0;
        CsrCacheStatus st = CsrCacheStatus::NotWritten;
        const CSR csr = cache ? loadTextCSRPathCached(argv[2], V, E, &st) : loadTextCSRPath(argv[1], V, E);
        if (cache) {
            std::cerr << (st == CsrCacheStatus::Hit       ? "cache: hit\n"
                          : st == CsrCacheStatus::Written ? "cache: written\n"
                                                          : "cache: not written\n");
        }
        uint64_t h = 1469598103934665603ULL;
        auto mix = [&h](int v) {
            const uint32_t u = static_cast<uint32_t>(v);
            for (int i = 0; i < 4; ++i) {
                h ^= (u >> (8 * i)) & 0xffu;
                h *= 1099511628211ULL;
            }
        };
        for (int v : csr.RowOffset) mix(v);
        for (int v : csr.ColInd) mix(v);
        std::printf("%d %d %016llx\n", V, E, static_cast<unsigned long long>(h));
    } catch (const std::exception& e) {
        std::cerr << e.what() << '\n';
        return 1;
    }
    return 0;
}
