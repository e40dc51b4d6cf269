// costWrite: calibrates the four operation weights on the B200 and saves them
// in the cost-file format cwlb-spmm reads (reference: weightCost.cpp:11-77).
//   costWrite
//   costWrite <K> <repeat> <WI> <load_MB> <atomic_writers>
//   costWrite --per-k <K1,K2,...> [<repeat> <WI> <load_MB> <atomic_writers>]
// Defaults: K=128, repeat=500, WI=131072, load_MB=512, atomic_writers=8.
// The output path defaults to the reference's ../resources/spmm_costs.txt and
// can be overridden with CWLB_COSTFILE; CWLB_DEVICE picks the GPU.
// --per-k (an extension) calibrates once per listed row width K and writes the
// per-K table (../resources/spmm_costs_per_k.txt, or CWLB_COSTFILE_PER_K)
// that cwlb-spmm uses with CWLB_COSTS_PER_K=1.
#include <cstdlib>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "config.h"
#include "cwlb_queue.h"
#include "utils.h"

namespace {

// "32,128,512" -> {32, 128, 512}; std::invalid_argument on anything else.
std::vector<int> parse_k_list(const std::string& s) {
    std::vector<int> ks;
    std::stringstream ss(s);
    std::string item;
    while (std::getline(ss, item, ',')) {
        size_t used = 0;
        int k = 0;
        try {
            k = std::stoi(item, &used);
        } catch (const std::exception&) {
            throw std::invalid_argument("bad K list: " + s);
        }
        if (used != item.size()) throw std::invalid_argument("bad K list: " + s);
        ks.push_back(k);
    }
    if (ks.empty()) throw std::invalid_argument("bad K list: " + s);
    return ks;
}

int per_k_main(int argc, char** argv) {
    int repeat = 500, WI = 131072, load_MB = 512, writers = 8;
    const std::vector<int> ks = parse_k_list(argv[2]);
    if (argc == 7) {
        repeat = std::stoi(argv[3]);
        WI = std::stoi(argv[4]);
        load_MB = std::stoi(argv[5]);
        writers = std::stoi(argv[6]);
    }
    for (int k : ks) {
        if (k <= 0) throw std::invalid_argument("All microbenchmark parameters must be positive.");
    }
    if (repeat <= 0 || WI <= 0 || load_MB <= 0 || writers <= 0) {
        throw std::invalid_argument("All microbenchmark parameters must be positive.");
    }
    cwlb::Queue q;
    std::vector<SpmmCostParams> table;
    for (int k : ks) {
        std::cout << "[measure_spmm_costs] K=" << k << '\n';
        SpmmCostParams c = measure_spmm_costs(q, k, repeat, WI, load_MB, writers);
        c.K = k;
        std::cout << "K " << k << ": C_compute_ns " << c.C_compute_ns << " C_load_ns "
                  << c.C_load_ns << " C_store_ns " << c.C_store_ns << " C_atomic_ns "
                  << c.C_atomic_ns << '\n';
        table.push_back(c);
    }
    const char* env = std::getenv("CWLB_COSTFILE_PER_K");
    const std::string path = env ? std::string(env) : COSTFILEPATH_PER_K;
    if (!save_costs_per_k(table, path)) {
        throw std::runtime_error("Failed to write per-K cost file: " + path);
    }
    std::cout << "Saved per-K cost parameters to: " << path << '\n';
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc >= 2 && std::string(argv[1]) == "--per-k") {
            if (argc != 3 && argc != 7) {
                std::cerr << "Usage:\n"
                          << "  ./costWrite --per-k K1,K2,... [repeat] [WI] [load_MB] "
                             "[atomic_writers]\n";
                return 1;
            }
            return per_k_main(argc, argv);
        }
        int K = 128, repeat = 500, WI = 131072, load_MB = 512, writers = 8;
        if (argc != 1 && argc != 6) {
            std::cerr << "Usage:\n"
                      << "  ./costWrite\n"
                      << "  ./costWrite [K] [repeat] [WI] [load_MB] [atomic_writers]\n";
            return 1;
        }
        if (argc == 6) {
            K = std::stoi(argv[1]);
            repeat = std::stoi(argv[2]);
            WI = std::stoi(argv[3]);
            load_MB = std::stoi(argv[4]);
            writers = std::stoi(argv[5]);
        }
        if (K <= 0 || repeat <= 0 || WI <= 0 || load_MB <= 0 || writers <= 0) {
            throw std::invalid_argument("All microbenchmark parameters must be positive.");
        }
        cwlb::Queue q;
        std::cout << "[measure_spmm_costs] begin\n";
        const SpmmCostParams c = measure_spmm_costs(q, K, repeat, WI, load_MB, writers);
        std::cout << "[measure_spmm_costs] end\n";
        std::cout << "device: " << q.name() << '\n'
                  << "C_compute_ns: " << c.C_compute_ns << '\n'
                  << "C_load_ns: " << c.C_load_ns << '\n'
                  << "C_store_ns: " << c.C_store_ns << '\n'
                  << "C_atomic_ns: " << c.C_atomic_ns << '\n';
        const char* env = std::getenv("CWLB_COSTFILE");
        const std::string path = env ? std::string(env) : COSTFILEPATH;
        if (!save_costs_one_per_line(c, path)) {
            throw std::runtime_error("Failed to write microbenchmark cost file: " + path);
        }
        std::cout << "Saved cost parameters to: " << path << '\n';
    } catch (const std::exception& e) {
        std::cerr << e.what() << '\n';
        return 1;
    }
    return 0;
}
