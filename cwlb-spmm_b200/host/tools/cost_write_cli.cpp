// costWrite: calibrates the four operation weights on the B200 and saves them
// in the cost-file format cwlb-spmm reads (reference: weightCost.cpp:11-77).
//   costWrite
//   costWrite <K> <repeat> <WI> <load_MB> <atomic_writers>
// Defaults: K=128, repeat=500, WI=131072, load_MB=512, atomic_writers=8.
// The output path defaults to the reference's ../resources/spmm_costs.txt and
// can be overridden with CWLB_COSTFILE; CWLB_DEVICE picks the GPU.
#include <cstdlib>
#include <iostream>
#include <stdexcept>
#include <string>

#include "config.h"
#include "cwlb_queue.h"
#include "utils.h"

int main(int argc, char** argv) {
    try {
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
