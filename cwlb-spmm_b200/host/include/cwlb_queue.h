#pragma once
// cwlb::Queue: one CUDA device and stream of the B200 library.  It takes the
// place of the reference's sycl::queue in every interface function.
#include <string>

#include "cwlb_spmm.h"

namespace cwlb {

// Throws the C++ exception matching a cwlb_status (std::invalid_argument,
// std::overflow_error, std::runtime_error), carrying cwlb_last_error().
void check(int status);

class Queue {
public:
    // Binds CUDA device `device` (the CWLB_DEVICE environment variable, if set,
    // chooses it when device < 0).
    explicit Queue(int device = -1);
    ~Queue();
    Queue(const Queue&) = delete;
    Queue& operator=(const Queue&) = delete;

    cwlb_ctx* ctx() const { return ctx_; }
    void wait();
    long max_work_group_size() const { return max_wg_; }
    int max_compute_units() const { return cus_; }
    const std::string& name() const { return name_; }

    // The queue used by interface functions whose reference signature has
    // no queue (costWeightedTaskPartitioning): one per host thread.
    static Queue& thread_default();

private:
    cwlb_ctx* ctx_ = nullptr;
    long max_wg_ = 0;
    int cus_ = 0;
    std::string name_;
};

}  // namespace cwlb
