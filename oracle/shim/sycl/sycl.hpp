// Host-only stand-in for the subset of SYCL 2020 that the CWLB-SpMM reference
// sources use (src/parallelMatrix.cpp, src/utils.cpp, main.cpp,
// weightCost.cpp).  TEST INFRASTRUCTURE ONLY: it lets g++ compile those
// unmodified files so their behaviour can be run on a CPU and used as the
// parity pin for the oracle.  It is never linked into the product library.
//
// Execution model:
//   * every submitted command runs synchronously on the calling thread;
//   * range<1> kernels run as a plain loop over ids;
//   * nd_range<1> kernels run one work-group at a time, each work-item as a
//     ucontext fiber; item.barrier() yields to a scheduler which resumes the
//     group only after every live work-item reached the barrier (the same
//     semantics a GPU work-group barrier gives a convergent kernel);
//   * USM allocations are plain host allocations; buffers alias host memory
//     (so their destructor's write-back is implicit);
//   * event profiling reports steady_clock nanoseconds around the command.
// The emulated device answers get_info queries from a table that the test
// bridge can change (max work-group size, sub-group sizes, local memory,
// compute units).
#pragma once

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include <ucontext.h>

namespace sycl {

namespace detail {
struct DeviceTable {
    std::size_t max_work_group_size = 1024;
    std::vector<std::size_t> sub_group_sizes{32};
    std::uint64_t local_mem_size = 49152;
    std::uint32_t max_compute_units = 80;
    std::string name = "cwlb-host-emulation";
};
inline DeviceTable& device_table() {
    static DeviceTable t;
    return t;
}
inline std::uint64_t now_ns() {
    return static_cast<std::uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(
            std::chrono::steady_clock::now().time_since_epoch())
            .count());
}
}  // namespace detail

namespace info {
namespace device {
struct max_work_group_size { using return_type = std::size_t; };
struct sub_group_sizes { using return_type = std::vector<std::size_t>; };
struct local_mem_size { using return_type = std::uint64_t; };
struct max_compute_units { using return_type = std::uint32_t; };
struct name { using return_type = std::string; };
}  // namespace device
namespace event_profiling {
struct command_start { using return_type = std::uint64_t; };
struct command_end { using return_type = std::uint64_t; };
}  // namespace event_profiling
}  // namespace info

namespace access {
enum class mode { read, write, read_write, discard_write };
enum class fence_space { local_space, global_space, global_and_local };
enum class address_space { global_space, local_space, generic_space };
}  // namespace access

enum class memory_order { relaxed, acquire, release, acq_rel, seq_cst };
enum class memory_scope { work_item, sub_group, work_group, device, system };

class device {
public:
    template <typename Param>
    typename Param::return_type get_info() const {
        const auto& t = detail::device_table();
        if constexpr (std::is_same_v<Param, info::device::max_work_group_size>) {
            return t.max_work_group_size;
        } else if constexpr (std::is_same_v<Param, info::device::sub_group_sizes>) {
            return t.sub_group_sizes;
        } else if constexpr (std::is_same_v<Param, info::device::local_mem_size>) {
            return t.local_mem_size;
        } else if constexpr (std::is_same_v<Param, info::device::max_compute_units>) {
            return t.max_compute_units;
        } else {
            static_assert(std::is_same_v<Param, info::device::name>, "unsupported query");
            return t.name;
        }
    }
};

inline int gpu_selector_v(const device&) { return 1; }

namespace property {
namespace queue {
struct enable_profiling {};
}  // namespace queue
}  // namespace property

class event {
public:
    event() = default;
    event(std::uint64_t s, std::uint64_t e) : start_(s), end_(e) {}
    void wait() const {}
    template <typename Param>
    std::uint64_t get_profiling_info() const {
        if constexpr (std::is_same_v<Param, info::event_profiling::command_start>) {
            return start_;
        } else {
            return end_;
        }
    }

private:
    std::uint64_t start_ = 0;
    std::uint64_t end_ = 0;
};

template <int D = 1>
class range {
public:
    range() { for (int i = 0; i < D; ++i) v_[i] = 0; }
    explicit range(std::size_t a) { static_assert(D == 1, "rank"); v_[0] = a; }
    range(std::size_t a, std::size_t b) { static_assert(D == 2, "rank"); v_[0] = a; v_[1] = b; }
    std::size_t operator[](int i) const { return v_[i]; }
    std::size_t size() const {
        std::size_t s = 1;
        for (int i = 0; i < D; ++i) s *= v_[i];
        return s;
    }

private:
    std::size_t v_[D];
};

template <int D = 1>
class id {
public:
    explicit id(std::size_t a) : v_(a) {}
    std::size_t operator[](int) const { return v_; }
    operator std::size_t() const { return v_; }

private:
    std::size_t v_;
};

template <int D = 1>
class nd_range {
public:
    nd_range(range<D> g, range<D> l) : global_(g), local_(l) {}
    range<D> get_global_range() const { return global_; }
    range<D> get_local_range() const { return local_; }

private:
    range<D> global_;
    range<D> local_;
};

namespace detail {

// One work-group's fibers.  Work-items yield to the scheduler at barriers.
struct FiberGroup {
    enum State { RUNNABLE, AT_BARRIER, DONE };
    ucontext_t sched{};
    std::vector<ucontext_t> ctx;
    std::vector<std::unique_ptr<char[]>> stacks;
    std::vector<int> state;
    std::size_t current = 0;
    const std::function<void(std::size_t)>* body = nullptr;
    static constexpr std::size_t kStack = 64 * 1024;

    void ensure(std::size_t n) {
        while (stacks.size() < n) stacks.emplace_back(new char[kStack]);
        ctx.resize(n);
        state.assign(n, RUNNABLE);
    }
};

inline FiberGroup*& current_group() {
    static thread_local FiberGroup* g = nullptr;
    return g;
}

inline void fiber_entry(int lo, int hi) {
    // Two 32-bit halves of the work-item index (makecontext passes ints).
    const std::size_t i = (static_cast<std::size_t>(static_cast<unsigned>(hi)) << 32) |
                          static_cast<unsigned>(lo);
    FiberGroup* g = current_group();
    (*g->body)(i);
    g->state[i] = FiberGroup::DONE;
    // Returning resumes uc_link (the scheduler).
}

inline void barrier_yield() {
    FiberGroup* g = current_group();
    if (g == nullptr) return;
    const std::size_t i = g->current;
    g->state[i] = FiberGroup::AT_BARRIER;
    swapcontext(&g->ctx[i], &g->sched);
}

// Run one work-group of `n` work-items to completion.
inline void run_group(std::size_t n, const std::function<void(std::size_t)>& body) {
    static thread_local FiberGroup fg;
    fg.ensure(n);
    fg.body = &body;
    FiberGroup* saved = current_group();
    current_group() = &fg;
    for (std::size_t i = 0; i < n; ++i) {
        getcontext(&fg.ctx[i]);
        fg.ctx[i].uc_stack.ss_sp = fg.stacks[i].get();
        fg.ctx[i].uc_stack.ss_size = FiberGroup::kStack;
        fg.ctx[i].uc_link = &fg.sched;
        makecontext(&fg.ctx[i], reinterpret_cast<void (*)()>(&fiber_entry), 2,
                    static_cast<int>(i & 0xffffffffu), static_cast<int>(i >> 32));
    }
    for (;;) {
        bool any_live = false;
        for (std::size_t i = 0; i < n; ++i) {
            if (fg.state[i] != FiberGroup::RUNNABLE) continue;
            fg.current = i;
            swapcontext(&fg.sched, &fg.ctx[i]);
        }
        for (std::size_t i = 0; i < n; ++i) {
            if (fg.state[i] == FiberGroup::AT_BARRIER) {
                fg.state[i] = FiberGroup::RUNNABLE;
                any_live = true;
            }
        }
        if (!any_live) break;
    }
    current_group() = saved;
}

}  // namespace detail

template <int D = 1>
class nd_item {
public:
    nd_item(std::size_t group, std::size_t lid, std::size_t lrange, std::size_t ngroups)
        : group_(group), lid_(lid), lrange_(lrange), ngroups_(ngroups) {}
    std::size_t get_group_linear_id() const { return group_; }
    std::size_t get_group(int) const { return group_; }
    std::size_t get_local_id(int) const { return lid_; }
    std::size_t get_local_range(int) const { return lrange_; }
    std::size_t get_global_id(int) const { return group_ * lrange_ + lid_; }
    std::size_t get_group_range(int) const { return ngroups_; }
    void barrier(access::fence_space = access::fence_space::global_and_local) const {
        detail::barrier_yield();
    }

private:
    std::size_t group_, lid_, lrange_, ngroups_;
};

class handler;

template <typename T, int D = 1>
class accessor {
public:
    accessor(T* p, range<D> r) : p_(p), r_(r) {}
    range<D> get_range() const { return r_; }
    template <int DD = D, std::enable_if_t<DD == 1, int> = 0>
    T& operator[](std::size_t i) const { return p_[i]; }
    template <int DD = D, std::enable_if_t<DD == 2, int> = 0>
    T* operator[](std::size_t i) const { return p_ + i * r_[1]; }
    T* get_pointer() const { return p_; }

private:
    T* p_;
    range<D> r_;
};

template <typename T, int D = 1>
class buffer {
public:
    buffer(const T* host, range<D> r) : p_(const_cast<T*>(host)), r_(r) {}
    buffer(T* host, range<D> r) : p_(host), r_(r) {}
    template <access::mode M = access::mode::read_write>
    accessor<T, D> get_access(handler&) {
        return accessor<T, D>(p_, r_);
    }
    range<D> get_range() const { return r_; }

private:
    T* p_;
    range<D> r_;
};

// Work-group local memory: one allocation per command, shared by the
// work-items of the (single) work-group that runs at a time.
template <typename T, int D = 1>
class local_accessor {
public:
    local_accessor(std::size_t n, handler&)
        : mem_(std::make_shared<std::vector<T>>(n)) {}
    T& operator[](std::size_t i) const { return (*mem_)[i]; }

private:
    std::shared_ptr<std::vector<T>> mem_;
};

class handler {
public:
    template <typename Name = void, typename F>
    void parallel_for(range<1> r, F f) {
        for (std::size_t i = 0; i < r[0]; ++i) f(id<1>(i));
    }

    template <typename Name = void, typename F>
    void parallel_for(nd_range<1> ndr, F f) {
        const std::size_t gsz = ndr.get_global_range()[0];
        const std::size_t lsz = ndr.get_local_range()[0];
        if (lsz == 0 || gsz % lsz != 0) {
            throw std::runtime_error("nd_range: global size not a multiple of local size");
        }
        const std::size_t groups = gsz / lsz;
        for (std::size_t g = 0; g < groups; ++g) {
            std::function<void(std::size_t)> body = [&](std::size_t lid) {
                f(nd_item<1>(g, lid, lsz, groups));
            };
            detail::run_group(lsz, body);
        }
    }
};

class queue {
public:
    queue() = default;
    template <typename Selector, typename... Props>
    explicit queue(const Selector&, Props...) {}

    device get_device() const { return device(); }

    template <typename Prop>
    bool has_property() const { return std::is_same_v<Prop, property::queue::enable_profiling>; }

    template <typename CGF>
    event submit(CGF cgf) {
        const std::uint64_t t0 = detail::now_ns();
        handler h;
        cgf(h);
        const std::uint64_t t1 = detail::now_ns();
        return event(t0, t1);
    }

    template <typename Name = void, typename F>
    event parallel_for(range<1> r, F f) {
        const std::uint64_t t0 = detail::now_ns();
        handler h;
        h.parallel_for<Name>(r, f);
        return event(t0, detail::now_ns());
    }

    template <typename Name = void, typename F>
    event parallel_for(nd_range<1> r, F f) {
        const std::uint64_t t0 = detail::now_ns();
        handler h;
        h.parallel_for<Name>(r, f);
        return event(t0, detail::now_ns());
    }

    event memcpy(void* dst, const void* src, std::size_t bytes) {
        if (bytes) std::memmove(dst, src, bytes);
        return event();
    }
    event memset(void* dst, int v, std::size_t bytes) {
        if (bytes) std::memset(dst, v, bytes);
        return event();
    }
    template <typename T>
    event fill(T* dst, const T& v, std::size_t count) {
        for (std::size_t i = 0; i < count; ++i) dst[i] = v;
        return event();
    }
    void wait() {}
};

template <typename T>
T* malloc_device(std::size_t n, const queue&) {
    return static_cast<T*>(std::calloc(n == 0 ? 1 : n, sizeof(T)));
}
template <typename T>
T* malloc_shared(std::size_t n, const queue&) {
    return static_cast<T*>(std::calloc(n == 0 ? 1 : n, sizeof(T)));
}
inline void free(void* p, const queue&) { std::free(p); }

template <typename T, memory_order O = memory_order::relaxed,
          memory_scope S = memory_scope::device,
          access::address_space A = access::address_space::generic_space>
class atomic_ref {
public:
    explicit atomic_ref(T& r) : p_(&r) {}
    T fetch_add(T v) const {
        // Single host thread executes work-items; a plain read-modify-write
        // is atomic with respect to them.
        T old = *p_;
        *p_ = old + v;
        return old;
    }
    T load() const { return *p_; }
    void store(T v) const { *p_ = v; }

private:
    T* p_;
};

template <typename T>
T fma(T a, T b, T c) { return std::fma(a, b, c); }

template <typename T>
T clamp(T x, T lo, T hi) { return std::min(std::max(x, lo), hi); }

}  // namespace sycl
