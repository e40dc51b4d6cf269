// cwlb::Queue and status-to-exception translation.
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "cwlb_queue.h"

namespace cwlb {

void check(int status) {
    if (status == CWLB_OK) return;
    const std::string msg = cwlb_last_error();
    switch (status) {
        case CWLB_ERR_INVALID_ARGUMENT: throw std::invalid_argument(msg);
        case CWLB_ERR_OVERFLOW: throw std::overflow_error(msg);
        default: throw std::runtime_error(msg);
    }
}

Queue::Queue(int device) {
    if (device < 0) {
        const char* env = std::getenv("CWLB_DEVICE");
        device = env ? std::atoi(env) : 0;
    }
    check(cwlb_ctx_create(device, &ctx_));
    int64_t mwg = 0, lmem = 0;
    int32_t cus = 0;
    char name[256] = {0};
    check(cwlb_device_info(ctx_, &mwg, &cus, &lmem, name, sizeof(name)));
    max_wg_ = static_cast<long>(mwg);
    cus_ = cus;
    name_ = name;
}

Queue::~Queue() {
    if (ctx_) cwlb_ctx_destroy(ctx_);
}

void Queue::wait() { check(cwlb_ctx_synchronize(ctx_)); }

Queue& Queue::thread_default() {
    static thread_local Queue q;
    return q;
}

}  // namespace cwlb
