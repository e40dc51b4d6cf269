// Host <-> device copies of caller memory for the host-buffer entry points.
//
// Memory the caller allocated with cudaHostAlloc / cudaHostRegister (pinned)
// is copied directly: the copy engines read it at PCIe speed (~55 GB/s on a
// B200 host).  Ordinary (pageable) memory is what the reference's callers
// pass (std::vector, numpy arrays); the driver copies it through its own
// bounce buffer at ~11 GB/s host -> device, and device -> host into pages the
// process has not touched yet (a freshly allocated result) at ~2 GB/s, because
// one thread takes every page fault.  Large pageable copies therefore go
// through a ring of pinned slots owned by the context, filled or drained by a
// pool of host threads while the copy engine moves the neighbouring slot:
//   host -> device: wait until slot k's previous transfer is done, copy the
//                   next piece of the caller's array into it (all pool threads),
//                   queue the DMA from the slot, record the slot's event;
//   device -> host: queue up to kSlots DMAs into slots ahead, then in order
//                   wait for each and copy it out to the caller (pool threads).
// Both return only when the caller's memory may be reused (host -> device) or
// holds the data (device -> host), as the driver's pageable copies do.
#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

namespace cwlb {

namespace {

constexpr size_t kDirectBytes = size_t(4) << 20;  // smaller copies: the driver's path
constexpr size_t kSlotBytes = size_t(32) << 20;
constexpr int kSlots = 4;
constexpr size_t kMinPart = size_t(2) << 20;  // bytes per pool thread, at least

// Threads that split one memcpy between them; the calling thread takes part 0.
class CopyPool {
public:
    explicit CopyPool(unsigned workers) {
        for (unsigned i = 0; i < workers; ++i) threads_.emplace_back([this, i] { loop(i + 1); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }
    void copy(void* dst, const void* src, size_t bytes) {
        const size_t most = threads_.size() + 1;
        const size_t parts = std::max<size_t>(1, std::min(most, bytes / kMinPart));
        if (parts == 1) {
            std::memcpy(dst, src, bytes);
            return;
        }
        {
            std::lock_guard<std::mutex> g(m_);
            dst_ = static_cast<char*>(dst);
            src_ = static_cast<const char*>(src);
            bytes_ = bytes;
            parts_ = parts;
            pending_ = parts - 1;
            ++gen_;
        }
        cv_.notify_all();
        part(0);
        std::unique_lock<std::mutex> lk(m_);
        done_.wait(lk, [this] { return pending_ == 0; });
    }

private:
    // Part p of the current job: 64-byte aligned boundaries.
    void part(size_t p) {
        const size_t per = (bytes_ / parts_) & ~size_t(63);
        const size_t b = p * per;
        const size_t e = p + 1 == parts_ ? bytes_ : b + per;
        std::memcpy(dst_ + b, src_ + b, e - b);
    }
    void loop(size_t idx) {
        uint64_t seen = 0;
        for (;;) {
            size_t parts;
            {
                std::unique_lock<std::mutex> lk(m_);
                cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
                parts = parts_;
            }
            if (idx < parts) {
                part(idx);
                std::lock_guard<std::mutex> g(m_);
                if (--pending_ == 0) done_.notify_one();
            }
        }
    }

    std::vector<std::thread> threads_;
    std::mutex m_;
    std::condition_variable cv_, done_;
    bool stop_ = false;
    uint64_t gen_ = 0;
    size_t pending_ = 0, parts_ = 1, bytes_ = 0;
    char* dst_ = nullptr;
    const char* src_ = nullptr;
};

bool is_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // not a CUDA-known pointer: pageable
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

}  // namespace

struct HostStager {
    void* slot[kSlots] = {};
    cudaEvent_t ev[kSlots] = {};  // last transfer through the slot
    int next = 0;
    CopyPool pool;
    HostStager()
        : pool(std::max(1u, std::min(16u, std::thread::hardware_concurrency())) - 1) {
        try {
            for (int k = 0; k < kSlots; ++k) {
                CWLB_CUDA(cudaHostAlloc(&slot[k], kSlotBytes, cudaHostAllocDefault));
                CWLB_CUDA(cudaEventCreateWithFlags(&ev[k], cudaEventDisableTiming));
            }
        } catch (...) {
            release();
            throw;
        }
    }
    ~HostStager() { release(); }
    void release() {
        for (int k = 0; k < kSlots; ++k) {
            if (ev[k]) cudaEventSynchronize(ev[k]);
            if (slot[k]) cudaFreeHost(slot[k]);
            if (ev[k]) cudaEventDestroy(ev[k]);
            slot[k] = nullptr;
            ev[k] = nullptr;
        }
    }
};

namespace {

HostStager& stager(cwlb_ctx* ctx) {
    if (!ctx->stager) ctx->stager = new HostStager();
    return *ctx->stager;
}

}  // namespace

void copy_to_device(cwlb_ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return;
    if (bytes < kDirectBytes || is_pinned(src)) {
        CWLB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s));
        return;
    }
    HostStager& st = stager(ctx);
    for (size_t off = 0; off < bytes; off += kSlotBytes) {
        const size_t n = std::min(kSlotBytes, bytes - off);
        const int k = st.next;
        st.next = (k + 1) % kSlots;
        CWLB_CUDA(cudaEventSynchronize(st.ev[k]));
        st.pool.copy(st.slot[k], static_cast<const char*>(src) + off, n);
        CWLB_CUDA(cudaMemcpyAsync(static_cast<char*>(dst) + off, st.slot[k], n,
                                  cudaMemcpyHostToDevice, s));
        CWLB_CUDA(cudaEventRecord(st.ev[k], s));
    }
}

void copy_to_host(cwlb_ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return;
    if (bytes < kDirectBytes || is_pinned(dst)) {
        CWLB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s));
        CWLB_CUDA(cudaStreamSynchronize(s));
        return;
    }
    HostStager& st = stager(ctx);
    const size_t n_pieces = (bytes + kSlotBytes - 1) / kSlotBytes;
    std::vector<int> slot_of(n_pieces);
    size_t drained = 0;
    auto drain = [&] {
        const size_t off = drained * kSlotBytes;
        const int k = slot_of[drained];
        CWLB_CUDA(cudaEventSynchronize(st.ev[k]));
        st.pool.copy(static_cast<char*>(dst) + off, st.slot[k], std::min(kSlotBytes, bytes - off));
        ++drained;
    };
    for (size_t i = 0; i < n_pieces; ++i) {
        if (i - drained == static_cast<size_t>(kSlots)) drain();
        const size_t off = i * kSlotBytes;
        const int k = st.next;
        st.next = (k + 1) % kSlots;
        slot_of[i] = k;
        CWLB_CUDA(cudaEventSynchronize(st.ev[k]));  // an earlier transfer through slot k
        CWLB_CUDA(cudaMemcpyAsync(st.slot[k], static_cast<const char*>(src) + off,
                                  std::min(kSlotBytes, bytes - off), cudaMemcpyDeviceToHost, s));
        CWLB_CUDA(cudaEventRecord(st.ev[k], s));
    }
    while (drained < n_pieces) drain();
}

void destroy_stager(cwlb_ctx* ctx) {
    delete ctx->stager;
    ctx->stager = nullptr;
}

}  // namespace cwlb
