// cwlb-spmm: the command-line driver of the CWLB-SpMM hot path on B200.
//
// Same command lines, checks, messages and output lines as the reference's
// cwlb-spmm (main.cpp:431-741):
//   cwlb-spmm <dataset> <K> <wave>                    S from the wave count
//   cwlb-spmm <dataset> <K> --S <S>                   fixed S
//   cwlb-spmm <dataset> <K> <S_begin> <S_max> <S_step> S sweep, appended to results
//   cwlb-spmm <dataset> <K> --candidates              three wave-based S values
//   cwlb-spmm <dataset> <K> --candidate-search [count] | --step <step>
// Paths default to the reference's (../resources/...), overridable with
// CWLB_DATASET_DIR, CWLB_COSTFILE and CWLB_RESULTS; CWLB_DEVICE picks the GPU.
//
// Extensions: CWLB_CSR_CACHE=1 loads the dataset through the binary cache
// beside the text file (data.h), CWLB_DETERMINISTIC=1 merges split rows in a
// fixed order (bit-reproducible outputs), CWLB_COSTS_PER_K=1 takes the costs
// from the per-K table (costWrite --per-k) entry nearest to K, and a trailing
// --verify checks every run's output with validate_custom_csr_result (absolute
// tolerance 1e-4) against a float64 aggregation of the UNSORTED CSR computed on
// the device (cwlb_spmm_mean_reference_device), and exits with status 1 on a
// mismatch.  Without them, output and exit status are the reference's.
//
// Each S run partitions on the GPU, uploads the reordered CSR, X and the tasks
// once, and times LOOPCOUNT aggregation launches with CUDA events (the first
// WARMUPCOUNT are warm-up), reporting the mean of the timed ones in
// microseconds, as the reference's event-profiled loop does (main.cpp:338-412).
#include <algorithm>
#include <array>
#include <cctype>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <limits>
#include <memory>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "config.h"
#include "cwlb_queue.h"
#include "data.h"
#include "parallelMatrix.h"
#include "utils.h"

namespace {

constexpr int kMaxSearchPoints = 10000;

std::string env_or(const char* name, const std::string& fallback) {
    const char* v = std::getenv(name);
    return v ? std::string(v) : fallback;
}

std::string cost_path() { return env_or("CWLB_COSTFILE", COSTFILEPATH); }
std::string results_path() { return env_or("CWLB_RESULTS", "../resources/results.txt"); }

std::array<int, 3> candidate_waves(uint64_t nnz) {
    int32_t w[3];
    cwlb_recommended_candidate_w(nnz, w);
    return {w[0], w[1], w[2]};
}

// positive_count, search_interval, grid_by_count, grid_by_step and
// ask_yes_no restate main.cpp:98-184 of hhx-C/CWLB-SpMM (integer grid
// formulas and a prompt loop whose output callers compare byte for byte).
// That code is Copyright (c) 2026, Hongxing He, Guanlin He and Chunlin Li,
// under the BSD 3-Clause License: redistribution and use in source and binary
// forms, with or without modification, are permitted provided that the
// copyright notice, this list of conditions and the disclaimer are retained;
// neither the names of the copyright holders nor of the contributors may be
// used to endorse or promote derived products without prior written
// permission.  THE SOFTWARE IS PROVIDED "AS IS", WITHOUT WARRANTY OF ANY KIND.
int positive_count(const std::string& text) {
    std::size_t used = 0;
    const int v = std::stoi(text, &used);
    if (used != text.size() || v <= 0) {
        throw std::invalid_argument("Search count/step must be a positive integer.");
    }
    return v;
}

// The neighbourhood around the best of three ascending S candidates.
std::pair<int, int> search_interval(const std::array<int, 3>& s, std::size_t best) {
    if (best >= s.size() || s[0] <= 0 || s[1] < s[0] || s[2] < s[1]) {
        throw std::invalid_argument("Invalid ordered candidate values or best index.");
    }
    int64_t lo = s[0], hi = s[2];
    if (best == 0) {
        lo = 2LL * s[0] - s[1];
        hi = s[1];
    } else if (best == 2) {
        lo = s[1];
        hi = 2LL * s[2] - s[1];
    }
    lo = std::max<int64_t>(1, lo);
    hi = std::min<int64_t>(std::numeric_limits<int>::max(), hi);
    return {static_cast<int>(lo), static_cast<int>(hi)};
}

std::vector<int> grid_by_count(int lo, int hi, int requested) {
    if (lo <= 0 || hi < lo || requested <= 0) {
        throw std::invalid_argument("Invalid search interval or point count.");
    }
    const int64_t width = static_cast<int64_t>(hi) - lo;
    const int count = static_cast<int>(std::min<int64_t>(requested, width + 1));
    if (count > kMaxSearchPoints) {
        throw std::invalid_argument("Search plan exceeds 10000 points; reduce the count.");
    }
    if (count == 1) return {static_cast<int>(lo + width / 2)};
    std::vector<int> v;
    for (int i = 0; i < count; ++i) {
        v.push_back(static_cast<int>(lo + (width * i + (count - 1) / 2) / (count - 1)));
    }
    return v;
}

std::vector<int> grid_by_step(int lo, int hi, int step) {
    if (lo <= 0 || hi < lo || step <= 0) throw std::invalid_argument("Invalid search interval or step.");
    const int64_t width = static_cast<int64_t>(hi) - lo;
    const int64_t count = width / step + 1 + (width % step != 0);
    if (count > kMaxSearchPoints) {
        throw std::invalid_argument("Search plan exceeds 10000 points; increase the step.");
    }
    std::vector<int> v;
    for (int64_t x = lo; x <= hi; x += step) v.push_back(static_cast<int>(x));
    if (v.back() != hi) v.push_back(hi);
    return v;
}

bool ask_yes_no() {
    std::string a;
    for (;;) {
        std::cout << "Continue CWLB-SpMM for these S values? (yes/no): " << std::flush;
        if (!std::getline(std::cin, a)) return false;
        const auto f = a.find_first_not_of(" \t\r\n");
        const auto l = a.find_last_not_of(" \t\r\n");
        a = f == std::string::npos ? "" : a.substr(f, l - f + 1);
        for (auto& ch : a) ch = static_cast<char>(std::tolower(static_cast<unsigned char>(ch)));
        if (a == "yes") return true;
        if (a == "no") return false;
        std::cout << "Please enter yes or no.\n";
    }
}

// X for the CLI: mt19937(42) and U[0,1) floats, row-major (main.cpp:324-336).
Defined::RowMajorMatrixXf features(int rows, int cols) {
    Defined::RowMajorMatrixXf x(rows, cols);
    std::mt19937 gen(42);
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    float* p = x.data();
    const int64_t n = static_cast<int64_t>(rows) * cols;
    for (int64_t i = 0; i < n; ++i) p[i] = dist(gen);
    return x;
}

template <typename T>
struct DeviceArray {
    T* p = nullptr;
    explicit DeviceArray(std::size_t n, const T* src = nullptr) {
        if (cudaMalloc(&p, sizeof(T) * std::max<std::size_t>(n, 1)) != cudaSuccess) {
            throw std::runtime_error("device allocation failed");
        }
        if (src && n && cudaMemcpy(p, src, sizeof(T) * n, cudaMemcpyHostToDevice) != cudaSuccess) {
            throw std::runtime_error("host to device copy failed");
        }
    }
    ~DeviceArray() {
        if (p) cudaFree(p);
    }
};

struct RunResult {
    int s = 0;
    double capacity = 0.0;
    std::size_t tasks = 0;
    double mean_us = 0.0;
    std::vector<double> samples;
};

// One partition + timing loop (run_single_s, main.cpp:338-412) at segment size s.
class RunnerBase {
public:
    virtual ~RunnerBase() = default;
    virtual RunResult run(int s, bool keep_samples) = 0;
};

void print_iteration(int it, const std::string& device, int K, double us) {
    const bool warm = it < WARMUPCOUNT;
    std::cout << std::fixed << std::setprecision(6) << (warm ? "[Warm-up " : "[Iteration ")
              << (warm ? it + 1 : it - WARMUPCOUNT + 1) << '/'
              << (warm ? WARMUPCOUNT : LOOPCOUNT - WARMUPCOUNT) << "] device=" << device
              << " K=" << K << " time=" << us << " us\n";
}

class Runner : public RunnerBase {
public:
    Runner(cwlb::Queue& q, const CSR_Order& g, const Defined::RowMajorMatrixXf& x, int K,
           const SpmmCostParams& costs, const CSR* verify_against = nullptr)
        : q_(q), g_(g), K_(K), costs_(costs), x_host_(x), verify_(verify_against),
          ro_(g.RowOffset.size(), g.RowOffset.data()),
          col_(g.ColInd.size(), g.ColInd.data()), val_(g.Value.size(), g.Value.data()),
          org_(g.Origin_local.size(), g.Origin_local.data()),
          x_(static_cast<std::size_t>(x.rows()) * x.cols(), x.data()),
          out_(static_cast<std::size_t>(x.rows()) * x.cols()), rows_(x.rows()) {
        cudaEventCreate(&e0_);
        cudaEventCreate(&e1_);
    }
    ~Runner() {
        cudaEventDestroy(e0_);
        cudaEventDestroy(e1_);
    }

    RunResult run(int s, bool keep_samples) override {
        RunResult r;
        r.s = s;
        r.capacity = capacity_from_s(s, costs_);
        const std::vector<ParallelDataWeighted> tasks =
            costWeightedTaskPartitioning(q_, g_, costs_, r.capacity);
        r.tasks = tasks.size();
        // The reference dispatches on the device's max work-group size
        // (main.cpp:359-365); its error behaviour is kept by the library.
        if (K_ > q_.max_work_group_size() && K_ <= 0) throw std::logic_error("unreachable");
        DeviceArray<ParallelDataWeighted> d_tasks(tasks.size(), tasks.data());
        const int n = static_cast<int>(g_.Origin_local.size());
        const int nnz = static_cast<int>(g_.ColInd.size());
        int64_t bad = 0, unc = 0, cov = 0;
        cwlb::check(cwlb_tasks_check(q_.ctx(), n, nnz, ro_.p,
                                     reinterpret_cast<const cwlb_task*>(d_tasks.p),
                                     static_cast<int64_t>(tasks.size()), &bad, &unc, &cov));
        uint32_t flags = (bad == 0 && unc == 0 && cov == 0) ? CWLB_ROWS_COVERED : 0u;
        const char* det = std::getenv("CWLB_DETERMINISTIC");
        if (det && std::string(det) == "1") flags |= CWLB_DETERMINISTIC;
        cudaStream_t st = static_cast<cudaStream_t>(cwlb_ctx_stream(q_.ctx()));
        double sum = 0.0;
        for (int it = 0; it < LOOPCOUNT; ++it) {
            double us = 0.0;
            if (K_ > 0 && !tasks.empty()) {
                cudaEventRecord(e0_, st);
                cwlb::check(cwlb_spmm_mean_device(q_.ctx(), n, nnz, ro_.p, col_.p, val_.p, org_.p,
                                                  x_.p, rows_, K_,
                                                  reinterpret_cast<const cwlb_task*>(d_tasks.p),
                                                  static_cast<int64_t>(tasks.size()), out_.p, flags));
                cudaEventRecord(e1_, st);
                cudaEventSynchronize(e1_);
                float ms = 0.0f;
                cudaEventElapsedTime(&ms, e0_, e1_);
                us = ms * 1e3;
            }
            print_iteration(it, q_.name(), K_, us);
            if (it >= WARMUPCOUNT) {
                sum += us;
                if (keep_samples) r.samples.push_back(us);
            }
        }
        uint32_t dev_err = 0;
        cwlb::check(cwlb_ctx_take_device_errors(q_.ctx(), &dev_err));
        if (dev_err) throw std::invalid_argument("invalid CSR or task indices detected on the device");
        r.mean_us = sum / static_cast<double>(LOOPCOUNT - WARMUPCOUNT);
        if (verify_) verify(s);
        return r;
    }

private:
    // Compares the last launch's output with the float64 device aggregation
    // of the unsorted CSR (computed once).
    void verify(int s) {
        const std::size_t n = static_cast<std::size_t>(rows_) * static_cast<std::size_t>(K_);
        if (reference_.rows() != rows_ || reference_.cols() != K_) {
            const CSR& c = *verify_;
            DeviceArray<int> ro(c.RowOffset.size(), c.RowOffset.data());
            DeviceArray<int> col(c.ColInd.size(), c.ColInd.data());
            DeviceArray<float> val(c.Value.size(), c.Value.data());
            DeviceArray<float> ref(n);
            cwlb::check(cwlb_spmm_mean_reference_device(
                q_.ctx(), static_cast<int32_t>(c.RowOffset.size()) - 1,
                static_cast<int32_t>(c.ColInd.size()), ro.p, col.p, val.p, x_.p, rows_, K_, ref.p));
            q_.wait();
            uint32_t dev_err = 0;
            cwlb::check(cwlb_ctx_take_device_errors(q_.ctx(), &dev_err));
            if (dev_err) throw std::invalid_argument("invalid CSR indices detected on the device");
            reference_ = Defined::RowMajorMatrixXf(rows_, K_);
            if (n && cudaMemcpy(reference_.data(), ref.p, sizeof(float) * n, cudaMemcpyDeviceToHost) !=
                         cudaSuccess) {
                throw std::runtime_error("device to host copy failed");
            }
        }
        Defined::RowMajorMatrixXf result(rows_, K_);
        if (n && cudaMemcpy(result.data(), out_.p, sizeof(float) * n, cudaMemcpyDeviceToHost) !=
                     cudaSuccess) {
            throw std::runtime_error("device to host copy failed");
        }
        std::cout << "[Verify] S=" << s << ' ';
        if (!validate_custom_csr_result(result, reference_, *verify_, x_host_, 1e-4f)) {
            throw std::runtime_error("Verification failed for S=" + std::to_string(s) + ".");
        }
    }

    cwlb::Queue& q_;
    const CSR_Order& g_;
    int K_;
    SpmmCostParams costs_;
    const Defined::RowMajorMatrixXf& x_host_;
    const CSR* verify_;
    Defined::RowMajorMatrixXf reference_;
    DeviceArray<int> ro_, col_;
    DeviceArray<float> val_;
    DeviceArray<int> org_;
    DeviceArray<float> x_, out_;
    long rows_;
    cudaEvent_t e0_{}, e1_{};
};

// CWLB_GPUS=N (N >= 2): the same loop over N GPUs of this node through the
// library's shard entry points (cwlb_shard_create / cwlb_shard_aggregate_device):
// GPU g sorts, partitions and aggregates the g-th cost-balanced block of
// original rows with X replicated; an iteration's time is the largest of the
// GPUs' event times (all GPUs launch before any is waited for).  Before the
// timing loop the cut is re-weighted by the measured shard times
// (cwlb_shard_bounds_rebalance; CWLB_REBALANCE=R rounds, default 4, 0 keeps
// the modelled cut).
class MultiRunner : public RunnerBase {
public:
    MultiRunner(const std::vector<int>& devices, const CSR& graph,
                const Defined::RowMajorMatrixXf& x, int K, const SpmmCostParams& costs,
                bool verify)
        : graph_(graph), x_host_(x), K_(K), verify_(verify), rows_(x.rows()) {
        costs_ = cwlb_costs{costs.C_compute_ns, costs.C_load_ns, costs.C_store_ns,
                            costs.C_atomic_ns, costs.K, costs.WI, costs.repeat,
                            costs.atomic_writers_per_addr};
        for (int dev : devices) gpus_.emplace_back(new Gpu(dev, x));
        name_ = gpus_[0]->q.name() + " x" + std::to_string(devices.size());
    }
    ~MultiRunner() override {
        for (auto& g : gpus_) drop_shard(*g);
    }

    RunResult run(int s, bool keep_samples) override {
        RunResult r;
        r.s = s;
        r.capacity = cwlb_capacity_from_s(s, &costs_);
        const int G = static_cast<int>(gpus_.size());
        const int32_t n = static_cast<int32_t>(graph_.RowOffset.size()) - 1;
        const char* det = std::getenv("CWLB_DETERMINISTIC");
        const uint32_t flags = (det && std::string(det) == "1") ? CWLB_DETERMINISTIC : 0u;
        // The modelled cut, then up to CWLB_REBALANCE (default 4) cuts
        // re-weighted by the GPUs' measured shard times; the fastest is kept.
        std::vector<int32_t> cut(static_cast<std::size_t>(G) + 1), best;
        cwlb::check(cwlb_shard_bounds(n, graph_.RowOffset.data(), &costs_, G, cut.data()));
        const char* rb = std::getenv("CWLB_REBALANCE");
        const int rounds = rb ? std::max(0, std::atoi(rb)) : 4;
        build(cut, r.capacity);
        double best_ms = 0.0;
        for (int k = 0; rounds > 0 && k <= rounds; ++k) {
            const std::vector<double> t = shard_ms(flags);
            const double worst = *std::max_element(t.begin(), t.end());
            if (best.empty() || worst < best_ms) {
                best = cut;
                best_ms = worst;
            }
            if (k == rounds) break;
            std::vector<int32_t> next(cut.size());
            cwlb::check(cwlb_shard_bounds_rebalance(n, graph_.RowOffset.data(), &costs_, G,
                                                    cut.data(), t.data(), next.data()));
            if (next == cut) break;
            cut = next;
            build(cut, r.capacity);
        }
        if (!best.empty() && best != cut) {
            cut = best;
            build(cut, r.capacity);
        }
        for (auto& dp : gpus_) {
            int64_t nt = 0;
            cwlb::check(cwlb_shard_info(dp->shard, nullptr, nullptr, nullptr, &nt, nullptr));
            r.tasks += static_cast<std::size_t>(nt);
        }
        double sum = 0.0;
        for (int it = 0; it < LOOPCOUNT; ++it) {
            for (auto& dp : gpus_) {
                Gpu& d = *dp;
                cudaSetDevice(d.dev);
                cudaEventRecord(d.e0, d.stream());
                cwlb::check(cwlb_shard_aggregate_device(d.shard, d.x->p, rows_, K_, d.out->p, flags));
                cudaEventRecord(d.e1, d.stream());
            }
            double us = 0.0;
            for (auto& dp : gpus_) {
                Gpu& d = *dp;
                cudaSetDevice(d.dev);
                cudaEventSynchronize(d.e1);
                float ms = 0.0f;
                cudaEventElapsedTime(&ms, d.e0, d.e1);
                us = std::max(us, 1e3 * ms);
            }
            print_iteration(it, name_, K_, us);
            if (it >= WARMUPCOUNT) {
                sum += us;
                if (keep_samples) r.samples.push_back(us);
            }
        }
        for (auto& dp : gpus_) {
            uint32_t dev_err = 0;
            cwlb::check(cwlb_ctx_take_device_errors(dp->q.ctx(), &dev_err));
            if (dev_err) throw std::invalid_argument("invalid CSR or task indices detected on the device");
        }
        r.mean_us = sum / static_cast<double>(LOOPCOUNT - WARMUPCOUNT);
        if (verify_) verify(s);
        return r;
    }

private:
    // Every GPU's shard of `cut` (cwlb_shard_create_cut) and its output rows.
    void build(const std::vector<int32_t>& cut, double capacity) {
        const int G = static_cast<int>(gpus_.size());
        const int32_t n = static_cast<int32_t>(graph_.RowOffset.size()) - 1;
        const int32_t nnz = static_cast<int32_t>(graph_.ColInd.size());
        for (int g = 0; g < G; ++g) {
            Gpu& d = *gpus_[g];
            drop_shard(d);
            cwlb::check(cwlb_shard_create_cut(d.q.ctx(), n, nnz, graph_.RowOffset.data(),
                                              graph_.ColInd.data(), graph_.Value.data(), &costs_,
                                              capacity, cut.data(), g, G, &d.shard));
            cwlb::check(cwlb_shard_info(d.shard, &d.row_begin, &d.row_end, nullptr, nullptr, nullptr));
            d.out.reset(new DeviceArrayOn<float>(d.dev, static_cast<std::size_t>(d.row_end - d.row_begin) * K_));
        }
    }
    // Mean time (ms) of 3 aggregations of every GPU's shard, after one
    // untimed; all GPUs run at once.
    std::vector<double> shard_ms(uint32_t flags) {
        std::vector<double> t;
        for (int rep = 0; rep < 2; ++rep) {
            for (auto& dp : gpus_) {
                Gpu& d = *dp;
                cudaSetDevice(d.dev);
                if (rep == 1) cudaEventRecord(d.e0, d.stream());
                for (int i = 0; i < (rep == 0 ? 1 : 3); ++i)
                    cwlb::check(cwlb_shard_aggregate_device(d.shard, d.x->p, rows_, K_, d.out->p, flags));
                if (rep == 1) cudaEventRecord(d.e1, d.stream());
            }
        }
        for (auto& dp : gpus_) {
            Gpu& d = *dp;
            cudaSetDevice(d.dev);
            cudaEventSynchronize(d.e1);
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, d.e0, d.e1);
            t.push_back(static_cast<double>(ms) / 3.0);
        }
        return t;
    }

    template <typename T>
    struct DeviceArrayOn {
        int dev;
        T* p = nullptr;
        DeviceArrayOn(int device, std::size_t n, const T* src = nullptr) : dev(device) {
            cudaSetDevice(dev);
            if (cudaMalloc(&p, sizeof(T) * std::max<std::size_t>(n, 1)) != cudaSuccess) {
                throw std::runtime_error("device allocation failed");
            }
            if (src && n && cudaMemcpy(p, src, sizeof(T) * n, cudaMemcpyHostToDevice) != cudaSuccess) {
                throw std::runtime_error("host to device copy failed");
            }
        }
        ~DeviceArrayOn() {
            cudaSetDevice(dev);
            if (p) cudaFree(p);
        }
    };
    struct Gpu {
        int dev;
        cwlb::Queue q;
        std::unique_ptr<DeviceArrayOn<float>> x, out;
        cwlb_shard* shard = nullptr;
        int32_t row_begin = 0, row_end = 0;
        cudaEvent_t e0{}, e1{};
        Gpu(int device, const Defined::RowMajorMatrixXf& xh) : dev(device), q(device) {
            x.reset(new DeviceArrayOn<float>(device, static_cast<std::size_t>(xh.rows()) * xh.cols(),
                                             xh.data()));
            cudaSetDevice(dev);
            cudaEventCreate(&e0);
            cudaEventCreate(&e1);
        }
        ~Gpu() {
            cudaSetDevice(dev);
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
        }
        cudaStream_t stream() const { return static_cast<cudaStream_t>(cwlb_ctx_stream(q.ctx())); }
    };
    static void drop_shard(Gpu& d) {
        if (d.shard) cwlb_shard_destroy(d.shard);
        d.shard = nullptr;
    }

    // The assembled output (each GPU's block of rows) against the float64
    // device aggregation of the unsorted CSR on the first GPU.
    void verify(int s) {
        const std::size_t nk = static_cast<std::size_t>(rows_) * static_cast<std::size_t>(K_);
        Defined::RowMajorMatrixXf result(rows_, K_);
        for (auto& dp : gpus_) {
            Gpu& d = *dp;
            cudaSetDevice(d.dev);
            const std::size_t b = static_cast<std::size_t>(d.row_end - d.row_begin) * K_;
            if (b && cudaMemcpy(result.data() + static_cast<std::size_t>(d.row_begin) * K_, d.out->p,
                                sizeof(float) * b, cudaMemcpyDeviceToHost) != cudaSuccess) {
                throw std::runtime_error("device to host copy failed");
            }
        }
        if (reference_.rows() != rows_ || reference_.cols() != K_) {
            Gpu& d = *gpus_[0];
            DeviceArrayOn<int> ro(d.dev, graph_.RowOffset.size(), graph_.RowOffset.data());
            DeviceArrayOn<int> col(d.dev, graph_.ColInd.size(), graph_.ColInd.data());
            DeviceArrayOn<float> val(d.dev, graph_.Value.size(), graph_.Value.data());
            DeviceArrayOn<float> ref(d.dev, nk);
            cwlb::check(cwlb_spmm_mean_reference_device(
                d.q.ctx(), static_cast<int32_t>(graph_.RowOffset.size()) - 1,
                static_cast<int32_t>(graph_.ColInd.size()), ro.p, col.p, val.p, d.x->p, rows_, K_,
                ref.p));
            d.q.wait();
            reference_ = Defined::RowMajorMatrixXf(rows_, K_);
            if (nk && cudaMemcpy(reference_.data(), ref.p, sizeof(float) * nk,
                                 cudaMemcpyDeviceToHost) != cudaSuccess) {
                throw std::runtime_error("device to host copy failed");
            }
        }
        std::cout << "[Verify] S=" << s << ' ';
        if (!validate_custom_csr_result(result, reference_, graph_, x_host_, 1e-4f)) {
            throw std::runtime_error("Verification failed for S=" + std::to_string(s) + ".");
        }
    }

    const CSR& graph_;
    const Defined::RowMajorMatrixXf& x_host_;
    int K_;
    bool verify_;
    long rows_;
    cwlb_costs costs_{};
    std::string name_;
    std::vector<std::unique_ptr<Gpu>> gpus_;
    Defined::RowMajorMatrixXf reference_;
};

void print_result(const std::string& ds, int V, int E, const SpmmCostParams& c, const RunResult& r) {
    std::cout << std::fixed << std::setprecision(6) << "Dataset: " << ds << '\n'
              << "V: " << V << ", E: " << E << '\n'
              << "SpMM time: " << r.mean_us << " us\n"
              << "costs: C_compute_ns=" << c.C_compute_ns << " C_load_ns=" << c.C_load_ns
              << " C_store_ns=" << c.C_store_ns << " C_atomic_ns=" << c.C_atomic_ns << '\n';
}

// Devices of the multi-GPU extension from CWLB_DEVICES (comma-separated
// ordinals) or CWLB_GPUS (a count: ordinals 0..N-1); one device by default.
std::vector<int> multi_gpu_devices() {
    int avail = 0;
    cudaGetDeviceCount(&avail);
    std::vector<int> devs;
    if (const char* list = std::getenv("CWLB_DEVICES")) {
        std::stringstream ss(list);
        std::string item;
        while (std::getline(ss, item, ',')) {
            int d = -1;
            try {
                d = std::stoi(item);
            } catch (const std::exception&) {
                d = -1;
            }
            if (d < 0 || d >= avail) {
                throw std::invalid_argument("CWLB_DEVICES must list device ordinals below " +
                                            std::to_string(avail) + ".");
            }
            devs.push_back(d);
        }
    } else if (const char* g = std::getenv("CWLB_GPUS")) {
        const int n = std::atoi(g);
        if (n < 1 || n > avail) {
            throw std::invalid_argument("CWLB_GPUS must be between 1 and the number of GPUs (" +
                                        std::to_string(avail) + ").");
        }
        for (int d = 0; d < n; ++d) devs.push_back(d);
    }
    if (devs.empty()) devs.push_back(0);
    return devs;
}

enum class Mode { Wave, FixedS, Sweep, Candidates, Search };

// Extension: `cwlb-spmm --dump-features ROWS COLS FILE` writes the X this
// CLI would use for a graph of ROWS vertices at K = COLS (features() above,
// float32, row-major, raw bytes) and exits; no device is touched.  Tests use
// it to compare the CLI's X bit for bit with the reference's.
int dump_features(int argc, char** argv) {
    if (argc != 5) throw std::invalid_argument("Usage: ./cwlb-spmm --dump-features ROWS COLS FILE");
    const int rows = std::stoi(argv[2]), cols = std::stoi(argv[3]);
    if (rows < 0 || cols < 0) throw std::invalid_argument("ROWS and COLS must not be negative.");
    const Defined::RowMajorMatrixXf x = features(rows, cols);
    std::ofstream f(argv[4], std::ios::binary | std::ios::trunc);
    if (!f) throw std::runtime_error(std::string("Cannot open ") + argv[4]);
    f.write(reinterpret_cast<const char*>(x.data()),
            static_cast<std::streamsize>(sizeof(float) * static_cast<std::size_t>(rows) * cols));
    if (!f) throw std::runtime_error(std::string("Cannot write ") + argv[4]);
    return 0;
}

int cli(int argc, char** argv) {
    if (argc > 1 && std::string(argv[1]) == "--dump-features") return dump_features(argc, argv);
    const bool verify = argc > 1 && std::string(argv[argc - 1]) == "--verify";
    if (verify) --argc;
    if (argc != 4 && argc != 5 && argc != 6) {
        std::cerr << "Usage:\n"
                  << "  ./cwlb-spmm [dataset] [K] [wave]\n"
                  << "  ./cwlb-spmm [dataset] [K] --S [S]\n"
                  << "  ./cwlb-spmm [dataset] [K] --candidates\n"
                  << "  ./cwlb-spmm [dataset] [K] --candidate-search [count=6]\n"
                  << "  ./cwlb-spmm [dataset] [K] --candidate-search --step [step]\n"
                  << "  ./cwlb-spmm [dataset] [K] [S_begin] [S_max] [S_step]\n";
        return 1;
    }
    const std::string ds = argv[1];
    const int K = std::stoi(argv[2]);
    Mode mode = Mode::Wave;
    int value = 0, s_max = 0, s_step = 0, count = 6, step = 0;
    const std::string a3 = argv[3];
    if (a3 == "--candidate-search") {
        mode = Mode::Search;
        if (argc == 5) {
            count = positive_count(argv[4]);
        } else if (argc == 6 && std::string(argv[4]) == "--step") {
            step = positive_count(argv[5]);
        } else if (argc != 4) {
            throw std::invalid_argument("Use --candidate-search [count] or --candidate-search --step step.");
        }
    } else if (argc == 4) {
        if (a3 == "--candidates") mode = Mode::Candidates;
        else value = std::stoi(a3);
    } else if (argc == 5 && a3 == "--S") {
        mode = Mode::FixedS;
        value = std::stoi(argv[4]);
    } else if (argc == 6) {
        mode = Mode::Sweep;
        value = std::stoi(a3);
        s_max = std::stoi(argv[4]);
        s_step = std::stoi(argv[5]);
    } else {
        throw std::invalid_argument("The five-argument form must use --S.");
    }
    const bool candidates = mode == Mode::Candidates || mode == Mode::Search;
    if (K <= 0 || (!candidates && value <= 0)) {
        throw std::invalid_argument("K and the hyperparameter must be positive.");
    }
    if (mode == Mode::Sweep && (s_max <= 0 || s_step <= 0)) {
        throw std::invalid_argument("S_begin, S_max and S_step must be positive.");
    }
    if (mode == Mode::Sweep && value > s_max) {
        throw std::invalid_argument("S_begin must not be greater than S_max.");
    }

    int V = 0, E = 0;
    const char* use_cache = std::getenv("CWLB_CSR_CACHE");
    const CSR graph = (use_cache && std::string(use_cache) == "1") ? loadDatasetToCSRCached(ds, V, E)
                                                                   : loadDatasetToCSR(ds, V, E);
    cwlb::Queue q;
    SpmmCostParams costs;
    const char* per_k = std::getenv("CWLB_COSTS_PER_K");
    if (per_k && std::string(per_k) == "1") {
        // Extension: the costs calibrated at the row width nearest to K.
        const std::string path = env_or("CWLB_COSTFILE_PER_K", COSTFILEPATH_PER_K);
        std::vector<SpmmCostParams> table;
        if (!read_costs_per_k(table, path) || table.empty()) {
            throw std::runtime_error("Cannot read per-K cost file: " + path +
                                     ". Run ./costWrite --per-k first.");
        }
        costs = costs_for_k(table, K);
        std::cerr << "costs: per-K table entry K=" << costs.K << " (" << path << ")\n";
    } else if (!read_costs_one_per_line(costs, cost_path())) {
        throw std::runtime_error("Cannot read microbenchmark cost file: " + cost_path() +
                                 ". Run ./costWrite first.");
    }
    const Defined::RowMajorMatrixXf X = features(V, K);
    const CSR_Order sorted = sortCSRByDegree(graph, q);
    // Extension: CWLB_GPUS=N runs every timing loop on GPUs 0..N-1 of this
    // node; CWLB_DEVICES=a,b,... names the devices instead (one shard each).
    const std::vector<int> devices = multi_gpu_devices();
    std::unique_ptr<RunnerBase> runner_p;
    if (devices.size() > 1) {
        runner_p.reset(new MultiRunner(devices, graph, X, K, costs, verify));
    } else {
        runner_p.reset(new Runner(q, sorted, X, K, costs, verify ? &graph : nullptr));
    }
    RunnerBase& runner = *runner_p;

    if (candidates) {
        const int cus = q.max_compute_units();
        const uint64_t nnz = sorted.RowOffset.empty() ? 0ULL : static_cast<uint64_t>(sorted.RowOffset.back());
        const std::array<int, 3> waves = candidate_waves(nnz);
        std::cout << "[Candidates] dataset=" << ds << " K=" << K << " NNZ=" << nnz
                  << " compute_units=" << cus << " warmup_launches=" << WARMUPCOUNT
                  << " timed_launches=" << LOOPCOUNT - WARMUPCOUNT << '\n';
        struct Cand {
            int id, w, s;
            double us;
        };
        std::vector<Cand> cand;
        std::size_t best = 0;
        for (std::size_t i = 0; i < waves.size(); ++i) {
            const int s = wave_based_s(sorted, cus, waves[i]);
            std::cout << "[Candidates] running S" << i + 1 << " w=" << waves[i] << " S=" << s << '\n';
            const RunResult r = runner.run(s, true);
            if (!std::isfinite(r.mean_us) || r.mean_us <= 0.0) {
                throw std::runtime_error("Invalid candidate kernel time.");
            }
            print_result(ds, V, E, costs, r);
            std::cout << "candidate_samples_us\tS" << i + 1;
            for (double x : r.samples) std::cout << '\t' << x;
            std::cout << '\n';
            cand.push_back({static_cast<int>(i + 1), waves[i], s, r.mean_us});
            if (r.mean_us < cand[best].us) best = i;
        }
        std::cout << "\n=== Candidate summary (SpMM kernel time, us) ===\n"
                  << "candidate\tw\tS\tSpMM_time_us\n";
        for (const Cand& c : cand) std::cout << 'S' << c.id << '\t' << c.w << '\t' << c.s << '\t' << c.us << '\n';
        const Cand& b = cand[best];
        std::cout << "Best among the three measured candidates: S" << b.id << " (w=" << b.w
                  << ", S=" << b.s << "), SpMM time=" << b.us << " us\n"
                  << "best_candidate=S" << b.id << " best_S=" << b.s
                  << " best_kernel_time_us=" << b.us << '\n';
        if (mode == Mode::Search) {
            const auto iv = search_interval({cand[0].s, cand[1].s, cand[2].s}, best);
            const std::vector<int> plan = step > 0 ? grid_by_step(iv.first, iv.second, step)
                                                   : grid_by_count(iv.first, iv.second, count);
            std::cout << "[Search plan] lower=" << iv.first << " upper=" << iv.second;
            if (step > 0) std::cout << " manual_step=" << step;
            else std::cout << " requested_count=" << count;
            std::cout << " actual_count=" << plan.size() << '\n' << "[Search plan] S values:";
            for (int s : plan) std::cout << ' ' << s;
            std::cout << '\n';
            if (!ask_yes_no()) {
                std::cout << "Search cancelled; results.txt unchanged.\n";
                return 0;
            }
            Cand overall = b;
            std::string source = "initial_candidate_S" + std::to_string(b.id);
            std::vector<Cand> found;
            for (std::size_t i = 0; i < plan.size(); ++i) {
                std::cout << "[Search] running P" << i + 1 << " S=" << plan[i] << '\n';
                const RunResult r = runner.run(plan[i], true);
                if (!std::isfinite(r.mean_us) || r.mean_us <= 0.0) {
                    throw std::runtime_error("Invalid search kernel time.");
                }
                print_result(ds, V, E, costs, r);
                std::cout << "search_samples_us\tP" << i + 1;
                for (double x : r.samples) std::cout << '\t' << x;
                std::cout << '\n';
                found.push_back({static_cast<int>(i + 1), 0, plan[i], r.mean_us});
                if (r.mean_us < overall.us) {
                    overall = found.back();
                    source = "search_P" + std::to_string(i + 1);
                }
            }
            std::ostringstream rec;
            rec << std::fixed << std::setprecision(6) << "cwlb-spmm-candidates\t" << ds << '\t' << K << '\n';
            for (const Cand& c : cand) rec << c.s << '\t' << c.us << '\n';
            rec << "cwlb-spmm-candidate-search\t" << ds << '\t' << K << '\n';
            for (const Cand& c : found) rec << c.s << '\t' << c.us << '\n';
            std::ofstream f(results_path(), std::ios::out | std::ios::app);
            if (!f) throw std::runtime_error("Cannot append search results to " + results_path());
            f << rec.str();
            f.flush();
            if (!f) throw std::runtime_error("Failed to save candidate-search results.");
            std::cout << "\n=== Search summary (SpMM kernel time, us) ===\n" << "point\tS\tSpMM_time_us\n";
            for (const Cand& c : found) std::cout << 'P' << c.id << '\t' << c.s << '\t' << c.us << '\n';
            std::cout << "Best among all evaluated initial/search configurations: S=" << overall.s
                      << ", SpMM time=" << overall.us << " us\n"
                      << "final_best_S=" << overall.s << " final_best_kernel_time_us=" << overall.us
                      << " source=" << source << '\n'
                      << "Results appended to " << results_path() << '\n';
        }
        return 0;
    }
    if (mode == Mode::Sweep) {
        std::ofstream f(results_path(), std::ios::out | std::ios::app);
        if (!f.is_open()) throw std::runtime_error("Cannot open S search result file: " + results_path());
        f << "cwlb-spmm\t" << ds << '\t' << K << '\n';
        f << std::fixed << std::setprecision(6);
        f.flush();
        int best_s = 0;
        double best_us = std::numeric_limits<double>::infinity();
        for (int64_t s = value; s <= s_max; s += s_step) {
            const RunResult r = runner.run(static_cast<int>(s), false);
            print_result(ds, V, E, costs, r);
            f << r.s << '\t' << r.mean_us << '\n';
            f.flush();
            if (!f) throw std::runtime_error("Failed to append S search result file: " + results_path());
            if (r.mean_us < best_us) {
                best_s = r.s;
                best_us = r.mean_us;
            }
        }
        std::cout << std::fixed << std::setprecision(6) << "best_S=" << best_s
                  << " best_kernel_time_us=" << best_us << '\n';
        return 0;
    }
    const int s = mode == Mode::Wave ? wave_based_s(sorted, q.max_compute_units(), value) : value;
    const RunResult r = runner.run(s, false);
    print_result(ds, V, E, costs, r);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        return cli(argc, argv);
    } catch (const std::exception& e) {
        std::cerr << e.what() << '\n';
        return 1;
    }
}
