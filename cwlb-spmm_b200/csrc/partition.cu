// Cost-weighted task partitioning on the GPU, bit-identical to
// costWeightedTaskPartitioning (src/utils.cpp:832-1021 of the reference).
//
// The reference is a sequential greedy over rows with a double accumulator.
// Its weights depend on a row only through the row's degree:
//   full_w(d)  = (Cc + Cl) * d + Cs        (a complete row, direct store)
//   chunk_w(n) = (Cc + Cl) * n + Ca        (a fragment, atomic write-back)
// and rows arrive degree-sorted, so the row sequence is a short list of RUNS
// of equal degree.  With Cc + Cl > 0, full_w is non-decreasing in the degree,
// so "short" rows (full_w <= capacity, packed whole) form a prefix of runs and
// "long" rows (cut into chunks of at most S nonzeros) the remaining suffix.
//
// Short runs.  Inside a run every row has the same weight w, so a bin that
// starts empty always takes the same number m of rows (the same double
// additions happen in the same order); bins inside a run are periodic.  A
// single walker thread therefore only simulates, per run, the bin that
// crosses into it, one fresh bin (to learn m) and the remainder: O(m) double
// additions per run instead of O(rows).
//
// Long runs.  After the first long row, the only state a long row hands to
// the next is one bit: "my last chunk absorbed your (deg % S) prefix".  For a
// row of degree d entered with bit x, the reference emits
//   c(x) = x ? (d - r)/S : ceil(d/S)            tasks (r = d % S),
// its last chunk weighs chunk_w(x ? S : d - (c(0)-1) S), and the next bit is
// the absorption test of src/utils.cpp:915-939 on that weight and the next
// row's degree.  Each bit map f is one of the four maps {0,1}->{0,1}, so
// f^3 = f and the bits inside a run follow x0, f(x0), f(f(x0)), f(x0), ...
// A run is thus summarised by a transfer map and a task count per entry bit;
// these compose associatively, and one CTA scans them in batches of 1024.
// The first long row takes the short region's open bin (the prefix-absorption
// of src/utils.cpp:879-912) and is simulated literally by the walker.
//
// The walker writes compact descriptors (one task, a periodic run of bins, a
// row's middle chunks, or a long run); an expansion kernel then writes every
// task in parallel.  All double arithmetic uses __dmul_rn / __dadd_rn /
// __dsub_rn so nothing is contracted into an FMA, matching the reference's
// baseline-x86-64 host build.
//
// Costs that are not finite, or Cc + Cl <= 0, break the monotone structure;
// those (and row sequences that are not degree-sorted) run a literal
// single-thread restatement of the reference loop instead.  No loop here
// waits on another thread; every loop is bounded by the input size.
#include <cmath>
#include <mutex>
#include <string>

#include "common.cuh"
#include "scan.cuh"

namespace cwlb {
namespace {

struct Params {
    double wCL, Cs, Ca, cap;
    int32_t S;
    int32_t n;
};

__device__ __forceinline__ double full_w(const Params& p, int32_t d) {
    return __dadd_rn(__dmul_rn(p.wCL, static_cast<double>(d)), p.Cs);
}
__device__ __forceinline__ double chunk_w(const Params& p, int32_t nnz) {
    return __dadd_rn(__dmul_rn(p.wCL, static_cast<double>(nnz)), p.Ca);
}

enum DescKind : int32_t { kSingle = 0, kPeriodic = 1, kChunks = 2, kLongRun = 3 };

// One compact descriptor; `base` is the index of its first task.
struct Desc {
    int64_t base;
    int32_t kind;
    int32_t a, b, c, d;  // kSingle: task fields; kPeriodic: p, m, q; kChunks: row, off, count
    int32_t e, f, g;     // kLongRun: a=s, b=L, c=deg, d=next deg (-1), e=x0, f=f tab, g=F tab
    int32_t pad;
};

// ---------------------------------------------------------------------------
// runs of equal degree

__global__ void run_flags_kernel(const int32_t* __restrict__ rowoff, int32_t n,
                                 int32_t* __restrict__ flags) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t d = rowoff[i + 1] - rowoff[i];
    flags[i] = (i == 0 || d != rowoff[i] - rowoff[i - 1]) ? 1 : 0;
}

__global__ void run_compact_kernel(const int32_t* __restrict__ rowoff, int32_t n,
                                   const int32_t* __restrict__ pos,
                                   int32_t* __restrict__ run_start, int32_t* __restrict__ n_runs) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t d = rowoff[i + 1] - rowoff[i];
    const bool start = (i == 0 || d != rowoff[i] - rowoff[i - 1]);
    if (start) run_start[pos[i]] = static_cast<int32_t>(i);
    if (i == n - 1) {
        const int32_t r = pos[i] + (start ? 1 : 0);
        *n_runs = r;
        run_start[r] = n;
    }
}

// ---------------------------------------------------------------------------
// long-run transfer maps

struct Fn {
    int32_t tab;  // bit x = image of x
    int64_t c0, c1;
};
__device__ __forceinline__ int ap(int32_t tab, int x) { return (tab >> x) & 1; }
__device__ __forceinline__ Fn fn_identity() { return Fn{2, 0, 0}; }
// A first, then B.
__device__ __forceinline__ Fn fn_then(const Fn& A, const Fn& B) {
    const int a0 = ap(A.tab, 0), a1 = ap(A.tab, 1);
    Fn r;
    r.tab = ap(B.tab, a0) | (ap(B.tab, a1) << 1);
    r.c0 = A.c0 + (a0 ? B.c1 : B.c0);
    r.c1 = A.c1 + (a1 ? B.c1 : B.c0);
    return r;
}

// Absorption test of the last chunk (weight acc) against the next row
// (degree dn, -1 if none), src/utils.cpp:915-939.
__device__ __forceinline__ int absorbs(const Params& p, double acc, int32_t dn) {
    if (acc >= p.cap) return 0;
    if (dn < 0) return 0;
    if (full_w(p, dn) <= p.cap) return 0;
    const int32_t r2 = dn % p.S;
    if (r2 == 0 || r2 >= dn) return 0;
    const double w = chunk_w(p, r2);
    const double rem = __dsub_rn(p.cap, acc);
    if (w > rem) return 0;
    return 1;
}

struct LongRun {
    int32_t s, L, d, dn;
    int64_t cnt[2];  // tasks per row for entry bit 0 / 1
    int32_t ftab, Ftab;
};

__device__ __forceinline__ void long_run_maps(const Params& p, LongRun& lr) {
    const int32_t d = lr.d;
    if (d <= 0) {
        lr.cnt[0] = lr.cnt[1] = 0;
        lr.ftab = lr.Ftab = 0;
        return;
    }
    const int64_t S = p.S;
    const int32_t r = d % p.S;
    const int64_t c0 = (static_cast<int64_t>(d) + S - 1) / S;
    const bool can1 = r != 0 && r < d;
    const int64_t c1 = can1 ? (static_cast<int64_t>(d) - r) / S : c0;
    lr.cnt[0] = c0;
    lr.cnt[1] = c1;
    const int32_t take0 = static_cast<int32_t>(static_cast<int64_t>(d) - (c0 - 1) * S);
    const int32_t take1 = can1 ? p.S : take0;
    const double acc0 = chunk_w(p, take0);
    const double acc1 = chunk_w(p, take1);
    lr.ftab = absorbs(p, acc0, d) | (absorbs(p, acc1, d) << 1);
    lr.Ftab = absorbs(p, acc0, lr.dn) | (absorbs(p, acc1, lr.dn) << 1);
}

__device__ __forceinline__ Fn long_run_fn(const LongRun& lr) {
    const int32_t L = lr.L;
    Fn r;
    int32_t tab = 0;
    int64_t c[2];
    for (int x = 0; x < 2; ++x) {
        const int x1 = ap(lr.ftab, x);
        const int x2 = ap(lr.ftab, x1);
        const int last = L == 1 ? x : ((L - 1) % 2 == 1 ? x1 : x2);
        tab |= ap(lr.Ftab, last) << x;
        c[x] = lr.cnt[x] + static_cast<int64_t>(L / 2) * lr.cnt[x1] +
               static_cast<int64_t>((L - 1) / 2) * lr.cnt[x2];
    }
    r.tab = tab;
    r.c0 = c[0];
    r.c1 = c[1];
    return r;
}

// ---------------------------------------------------------------------------
// the walker: one CTA

constexpr int kWalkThreads = 1024;

struct WalkOut {
    int64_t n_tasks;
    int32_t n_desc;
    int32_t fallback;  // 1: structure not as assumed, use the literal path
};

__device__ __forceinline__ int32_t run_degree(const int32_t* rowoff, const int32_t* run_start,
                                              int32_t ri) {
    const int32_t s = run_start[ri];
    return rowoff[s + 1] - rowoff[s];
}

__global__ void __launch_bounds__(kWalkThreads)
    walk_kernel(Params p, const int32_t* __restrict__ rowoff,
                const int32_t* __restrict__ run_start, const int32_t* __restrict__ n_runs_ptr,
                Desc* __restrict__ desc, WalkOut* __restrict__ out) {
    __shared__ int32_t s_D, s_first_long_run, s_bit, s_first_entry_row, s_fallback;
    __shared__ int64_t s_T;
    const int32_t R = *n_runs_ptr;
    const int32_t n = p.n;

    if (threadIdx.x == 0) {
        int64_t T = 0;
        int32_t D = 0;
        auto single = [&](int32_t s, int32_t e, int32_t fo, int32_t last) {
            if (s < e) {
                Desc& q = desc[D++];
                q.base = T;
                q.kind = kSingle;
                q.a = s;
                q.b = e;
                q.c = fo;
                q.d = last;
                T += 1;
            }
        };
        int32_t g_start = 0, first_off = 0;
        double acc = 0.0;
        int32_t ri = 0;
        // ---------------- short runs ----------------
        for (; ri < R; ++ri) {
            const int32_t s = run_start[ri], e = run_start[ri + 1];
            const int32_t deg = rowoff[s + 1] - rowoff[s];
            const double w = full_w(p, deg);
            if (!(w <= p.cap)) break;
            int32_t row = s;
            while (row < e) {
                if (acc != 0.0) {
                    // finish the open bin
                    if (w == 0.0) {  // acc + 0 == acc: every row of the run fits
                        if (acc <= p.cap) {
                            row = e;
                            break;
                        }
                    }
                    while (row < e && (acc == 0.0 || __dadd_rn(acc, w) <= p.cap)) {
                        acc = __dadd_rn(acc, w);
                        ++row;
                    }
                    if (row < e) {
                        single(g_start, row, first_off, 0);
                        g_start = row;
                        first_off = 0;
                        acc = 0.0;
                    }
                    continue;
                }
                // a fresh bin starts at row (rows g_start..row-1 weigh zero)
                const int32_t left = e - row;
                if (w == 0.0) {  // zero-weight rows never close a bin
                    row = e;
                    break;
                }
                double a = 0.0;
                int32_t m = 0;
                while (m < left && (a == 0.0 || __dadd_rn(a, w) <= p.cap)) {
                    a = __dadd_rn(a, w);
                    ++m;
                }
                if (m == left && (a == 0.0 || __dadd_rn(a, w) <= p.cap)) {
                    acc = a;  // still open at the end of the run
                    row = e;
                    break;
                }
                // Every bin here holds exactly m rows.  A bin is closed only by
                // a following row of this run; one that ends exactly at the run
                // end stays open, because the next run's first row decides.
                const int32_t q = left / m;
                const int32_t rem = left - q * m;
                const int32_t closed = rem > 0 ? q : q - 1;
                if (closed >= 1) {
                    single(g_start, row + m, first_off, 0);
                    if (closed > 1) {
                        Desc& dd = desc[D++];
                        dd.base = T;
                        dd.kind = kPeriodic;
                        dd.a = row + m;
                        dd.b = m;
                        dd.c = closed - 1;
                        T += closed - 1;
                    }
                    row += closed * m;
                    g_start = row;
                    first_off = 0;
                    acc = 0.0;
                }
                for (int32_t k = row; k < e; ++k) acc = __dadd_rn(acc, w);
                row = e;
            }
        }
        int32_t bit = 0;
        int32_t first_entry_row = n;
        if (ri < R) {
            // ---------------- the first long row ----------------
            const int32_t L0 = run_start[ri];
            const int32_t e0 = run_start[ri + 1];
            const int32_t deg = rowoff[L0 + 1] - rowoff[L0];
            const bool absorbed = (acc == 0.0 && g_start == L0 && first_off > 0);
            int32_t off = absorbed ? first_off : 0;
            int32_t remaining = deg - off;
            if (remaining <= 0) {
                g_start = L0 + 1;
                first_off = 0;
                acc = 0.0;
            } else {
                if (!absorbed && !(acc <= 0.0)) {
                    const int32_t r = deg % p.S;
                    if (r == 0 || r >= deg) {
                        single(g_start, L0, first_off, 0);
                        g_start = L0;
                        first_off = 0;
                        acc = 0.0;
                    } else if (chunk_w(p, r) <= __dsub_rn(p.cap, acc)) {
                        single(g_start, L0 + 1, first_off, r);
                        g_start = L0;
                        first_off = r;
                        acc = 0.0;
                        remaining -= r;
                        off += r;
                    } else {
                        single(g_start, L0, first_off, 0);
                        g_start = L0;
                        first_off = 0;
                        acc = 0.0;
                    }
                }
                // chunk 0
                int32_t take = min(remaining, p.S);
                acc = __dadd_rn(acc, chunk_w(p, take));
                remaining -= take;
                off += take;
                if (remaining > 0) {
                    single(g_start, L0 + 1, first_off, off);
                    g_start = L0;
                    first_off = off;
                    acc = 0.0;
                    // middle chunks: every one emits (L0, L0+1, off, off+S)
                    const int32_t mid = (remaining - 1) / p.S;
                    if (mid > 0) {
                        Desc& dd = desc[D++];
                        dd.base = T;
                        dd.kind = kChunks;
                        dd.a = L0;
                        dd.b = off;
                        dd.c = mid;
                        T += mid;
                        off += mid * p.S;
                        remaining -= mid * p.S;
                        first_off = off;
                    }
                    // last chunk
                    take = remaining;
                    acc = __dadd_rn(0.0, chunk_w(p, take));
                    remaining = 0;
                    off += take;
                }
                // absorption of the next row's prefix
                const int32_t dn = L0 + 1 < n ? rowoff[L0 + 2] - rowoff[L0 + 1] : -1;
                if (dn >= 0 && absorbs(p, acc, dn)) {
                    single(g_start, L0 + 2, first_off, dn % p.S);
                    g_start = L0 + 1;
                    first_off = dn % p.S;
                    acc = 0.0;
                } else {
                    single(g_start, L0 + 1, first_off, 0);
                    g_start = L0 + 1;
                    first_off = 0;
                    acc = 0.0;
                }
            }
            bit = first_off > 0 ? 1 : 0;
            first_entry_row = L0 + 1;
            s_first_long_run = (L0 + 1 < e0) ? ri : ri + 1;  // entry 0 = rest of this run
        } else {
            // no long rows: final flush (src/utils.cpp:1016-1018)
            if (acc > 0.0 || g_start < n) single(g_start, n, first_off, 0);
            s_first_long_run = R;
        }
        s_T = T;
        s_D = D;
        s_bit = bit;
        s_first_entry_row = first_entry_row;
        s_fallback = 0;
    }
    __syncthreads();

    // ---------------- long entries: block scan of transfer maps ----------------
    const int32_t r_first = s_first_long_run;
    const int32_t row0 = s_first_entry_row;
    const int32_t n_entries = R - r_first;
    __shared__ int32_t w_tab[kWalkThreads / 32];
    __shared__ int64_t w_c0[kWalkThreads / 32], w_c1[kWalkThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int32_t e0 = 0; e0 < n_entries; e0 += kWalkThreads) {
        const int32_t ei = e0 + threadIdx.x;
        const bool valid = ei < n_entries;
        LongRun lr{};
        Fn mine = fn_identity();
        if (valid) {
            const int32_t ri = r_first + ei;
            lr.s = max(run_start[ri], row0);
            lr.L = run_start[ri + 1] - lr.s;
            lr.d = run_degree(rowoff, run_start, ri);
            lr.dn = ri + 1 < R ? run_degree(rowoff, run_start, ri + 1) : -1;
            if (!(full_w(p, lr.d) > p.cap)) s_fallback = 1;  // a short row after long rows
            long_run_maps(p, lr);
            mine = long_run_fn(lr);
        }
        // inclusive warp scan
        Fn inc = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            Fn prev;
            prev.tab = __shfl_up_sync(0xffffffffu, inc.tab, o);
            prev.c0 = __shfl_up_sync(0xffffffffu, inc.c0, o);
            prev.c1 = __shfl_up_sync(0xffffffffu, inc.c1, o);
            if (lane >= o) inc = fn_then(prev, inc);
        }
        if (lane == 31) {
            w_tab[warp] = inc.tab;
            w_c0[warp] = inc.c0;
            w_c1[warp] = inc.c1;
        }
        __syncthreads();
        if (warp == 0) {
            Fn x{w_tab[lane], w_c0[lane], w_c1[lane]};
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                Fn prev;
                prev.tab = __shfl_up_sync(0xffffffffu, x.tab, o);
                prev.c0 = __shfl_up_sync(0xffffffffu, x.c0, o);
                prev.c1 = __shfl_up_sync(0xffffffffu, x.c1, o);
                if (lane >= o) x = fn_then(prev, x);
            }
            w_tab[lane] = x.tab;  // inclusive over warps
            w_c0[lane] = x.c0;
            w_c1[lane] = x.c1;
        }
        __syncthreads();
        // exclusive prefix of this entry = (warps before) then (lanes before)
        Fn excl = warp > 0 ? Fn{w_tab[warp - 1], w_c0[warp - 1], w_c1[warp - 1]} : fn_identity();
        Fn lane_ex;
        lane_ex.tab = __shfl_up_sync(0xffffffffu, inc.tab, 1);
        lane_ex.c0 = __shfl_up_sync(0xffffffffu, inc.c0, 1);
        lane_ex.c1 = __shfl_up_sync(0xffffffffu, inc.c1, 1);
        if (lane == 0) lane_ex = fn_identity();
        excl = fn_then(excl, lane_ex);
        const int carry_bit = s_bit;
        const int64_t carry_T = s_T;
        if (valid) {
            const int x0 = ap(excl.tab, carry_bit);
            const int64_t base = carry_T + (carry_bit ? excl.c1 : excl.c0);
            Desc& dd = desc[s_D + ei];
            dd.base = base;
            dd.kind = kLongRun;
            dd.a = lr.s;
            dd.b = lr.L;
            dd.c = lr.d;
            dd.d = lr.dn;
            dd.e = x0;
            dd.f = lr.ftab;
            dd.g = lr.Ftab;
            // per-row task counts are recomputed by the expander from d and S
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            const Fn tot{w_tab[kWalkThreads / 32 - 1], w_c0[kWalkThreads / 32 - 1],
                         w_c1[kWalkThreads / 32 - 1]};
            s_T = carry_T + (carry_bit ? tot.c1 : tot.c0);
            s_bit = ap(tot.tab, carry_bit);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        out->n_tasks = s_T;
        out->n_desc = s_D + max(n_entries, 0);
        out->fallback = s_fallback;
    }
}

// ---------------------------------------------------------------------------
// expansion: one thread per task

__global__ void expand_kernel(Params p, const Desc* __restrict__ desc, int32_t n_desc,
                              int64_t n_tasks, cwlb_task* __restrict__ tasks) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n_tasks) return;
    int32_t lo = 0, hi = n_desc;  // last descriptor with base <= t
    while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if (desc[mid].base <= t) lo = mid;
        else hi = mid;
    }
    const Desc& q = desc[lo];
    const int64_t u = t - q.base;
    cwlb_task out;
    if (q.kind == kSingle) {
        out = cwlb_task{q.a, q.b, q.c, q.d};
    } else if (q.kind == kPeriodic) {
        const int32_t s = q.a + static_cast<int32_t>(u) * q.b;
        out = cwlb_task{s, s + q.b, 0, 0};
    } else if (q.kind == kChunks) {
        const int32_t o = q.b + static_cast<int32_t>(u) * p.S;
        out = cwlb_task{q.a, q.a + 1, o, o + p.S};
    } else {
        const int32_t d = q.c, L = q.b, S = p.S;
        const int32_t r = d % S;
        const int64_t c0 = (static_cast<int64_t>(d) + S - 1) / S;
        const int64_t c1 = (r != 0 && r < d) ? (static_cast<int64_t>(d) - r) / S : c0;
        const int x0 = q.e;
        const int x1 = ap(q.f, x0);
        const int x2 = ap(q.f, x1);
        const int64_t n0 = x0 ? c1 : c0;
        const int64_t n1 = x1 ? c1 : c0;
        const int64_t n2 = x2 ? c1 : c0;
        int64_t j, k;
        int x;
        if (u < n0) {
            j = 0;
            k = u;
            x = x0;
        } else {
            const int64_t v = u - n0;
            const int64_t P = n1 + n2;
            const int64_t pair = v / P;
            const int64_t rem = v - pair * P;
            if (rem < n1) {
                j = 1 + 2 * pair;
                k = rem;
                x = x1;
            } else {
                j = 2 + 2 * pair;
                k = rem - n1;
                x = x2;
            }
        }
        const int32_t i = q.a + static_cast<int32_t>(j);
        const int64_t c = x ? c1 : c0;
        const int32_t off0 = x ? r : 0;
        const int32_t o = off0 + static_cast<int32_t>(k) * S;
        if (k < c - 1) {
            out = cwlb_task{i, i + 1, o, o + S};
        } else {
            const bool in_run = j < L - 1;
            const int y = in_run ? ap(q.f, x) : ap(q.g, x);
            const int32_t dnext = in_run ? d : q.d;
            if (y) out = cwlb_task{i, i + 2, o, dnext % S};
            else out = cwlb_task{i, i + 1, o, 0};
        }
    }
    tasks[t] = out;
}

// ---------------------------------------------------------------------------
// literal restatement (non-finite costs, Cc + Cl <= 0, unsorted rows)

__global__ void literal_partition_kernel(Params p, const int32_t* __restrict__ rp,
                                         cwlb_task* __restrict__ tasks, int64_t max_tasks,
                                         int64_t* __restrict__ n_out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int32_t n = p.n;
    int64_t count = 0;
    int32_t g_start = 0, first_off = 0, row = 0;
    double acc = 0.0;
    auto emit = [&](int32_t s, int32_t e, int32_t fo, int32_t last) {
        if (s >= e) return;
        if (tasks && count < max_tasks) tasks[count] = cwlb_task{s, e, fo, last};
        ++count;
    };
    while (row < n) {
        const int32_t deg = rp[row + 1] - rp[row];
        const double wr = full_w(p, deg);
        if (wr <= p.cap) {
            if (acc == 0.0 || __dadd_rn(acc, wr) <= p.cap) {
                acc = __dadd_rn(acc, wr);
                ++row;
            } else {
                emit(g_start, row, first_off, 0);
                g_start = row;
                first_off = 0;
                acc = 0.0;
            }
            continue;
        }
        const bool absorbed = (acc == 0.0 && g_start == row && first_off > 0);
        int32_t off = absorbed ? first_off : 0;
        int32_t remaining = deg - off;
        if (remaining <= 0) {
            g_start = row + 1;
            first_off = 0;
            acc = 0.0;
            ++row;
            continue;
        }
        if (!absorbed && !(acc <= 0.0)) {
            const int32_t r = deg % p.S;
            if (r == 0 || r >= deg) {
                emit(g_start, row, first_off, 0);
                g_start = row;
                first_off = 0;
                acc = 0.0;
            } else if (chunk_w(p, r) <= __dsub_rn(p.cap, acc)) {
                emit(g_start, row + 1, first_off, r);
                g_start = row;
                first_off = r;
                acc = 0.0;
                remaining -= r;
                off += r;
            } else {
                emit(g_start, row, first_off, 0);
                g_start = row;
                first_off = 0;
                acc = 0.0;
            }
        }
        while (remaining > 0) {
            const int32_t take = min(remaining, p.S);
            acc = __dadd_rn(acc, chunk_w(p, take));
            remaining -= take;
            off += take;
            if (remaining > 0) {
                emit(g_start, row + 1, first_off, off);
                g_start = row;
                first_off = off;
                acc = 0.0;
                continue;
            }
            bool took = false;
            if (!(acc >= p.cap) && row + 1 < n) {
                const int32_t nr = row + 1;
                const int32_t nd = rp[nr + 1] - rp[nr];
                if (!(full_w(p, nd) <= p.cap)) {
                    const int32_t r2 = nd % p.S;
                    if (!(r2 == 0 || r2 >= nd)) {
                        const double w = chunk_w(p, r2);
                        const double rem = __dsub_rn(p.cap, acc);
                        if (!(w > rem)) {
                            emit(g_start, nr + 1, first_off, r2);
                            g_start = nr;
                            first_off = r2;
                            acc = 0.0;
                            took = true;
                        }
                    }
                }
            }
            if (!took) {
                emit(g_start, row + 1, first_off, 0);
                g_start = row + 1;
                first_off = 0;
                acc = 0.0;
            }
        }
        ++row;
    }
    if (acc > 0.0 || g_start < n) emit(g_start, n, first_off, 0);
    *n_out = count;
}

Params make_params(int32_t n_rows, const cwlb_costs& c, double capacity) {
    Params p;
    p.wCL = c.C_compute_ns + c.C_load_ns;
    p.Cs = c.C_store_ns;
    p.Ca = c.C_atomic_ns;
    p.cap = capacity;
    p.S = cwlb_segment_size(&c, capacity);
    p.n = n_rows;
    return p;
}

int64_t literal_partition(cwlb_ctx* ctx, const Params& p, const int32_t* d_rowoff) {
    cudaStream_t s = ctx->stream;
    int64_t* d_n = static_cast<int64_t*>(ctx->part_scratch.ensure(256));
    literal_partition_kernel<<<1, 32, 0, s>>>(p, d_rowoff, nullptr, 0, d_n);
    CWLB_LAUNCH_CHECK("literal_partition_kernel");
    int64_t cnt = 0;
    CWLB_CUDA(cudaMemcpyAsync(&cnt, d_n, sizeof(cnt), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    cwlb_task* d_tasks = ctx->part_tasks.as<cwlb_task>(static_cast<size_t>(cnt > 0 ? cnt : 1));
    literal_partition_kernel<<<1, 32, 0, s>>>(p, d_rowoff, d_tasks, cnt, d_n);
    CWLB_LAUNCH_CHECK("literal_partition_kernel");
    return cnt;
}

}  // namespace

int64_t run_partition(cwlb_ctx* ctx, int32_t n_rows, const int32_t* d_rowoff,
                      const cwlb_costs& costs, double capacity) {
    if (n_rows <= 0) return 0;
    const Params p = make_params(n_rows, costs, capacity);
    const bool fast = std::isfinite(p.wCL) && std::isfinite(p.Cs) && std::isfinite(p.Ca) &&
                      std::isfinite(p.cap) && p.wCL > 0.0;
    if (!fast) return literal_partition(ctx, p, d_rowoff);

    cudaStream_t s = ctx->stream;
    const int64_t n = n_rows;
    auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    const size_t b_flags = al(sizeof(int32_t) * n);
    const size_t b_scan = al(scan_scratch_bytes<int32_t>(n));
    const size_t b_runs = al(sizeof(int32_t) * (n + 1));
    char* base = static_cast<char*>(ctx->part_scratch.ensure(2 * b_flags + b_scan + b_runs + 512));
    int32_t* flags = reinterpret_cast<int32_t*>(base);
    int32_t* pos = reinterpret_cast<int32_t*>(base + b_flags);
    void* scan_tmp = base + 2 * b_flags;
    int32_t* run_start = reinterpret_cast<int32_t*>(base + 2 * b_flags + b_scan);
    int32_t* d_R = reinterpret_cast<int32_t*>(base + 2 * b_flags + b_scan + b_runs);

    const unsigned blocks = static_cast<unsigned>(ceil_div(n, 256));
    run_flags_kernel<<<blocks, 256, 0, s>>>(d_rowoff, n_rows, flags);
    CWLB_LAUNCH_CHECK("run_flags_kernel");
    device_exclusive_scan<int32_t>(flags, pos, n, scan_tmp, s);
    run_compact_kernel<<<blocks, 256, 0, s>>>(d_rowoff, n_rows, pos, run_start, d_R);
    CWLB_LAUNCH_CHECK("run_compact_kernel");
    int32_t R = 0;
    CWLB_CUDA(cudaMemcpyAsync(&R, d_R, sizeof(R), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));

    // Descriptors: <= 3 per short run, <= 4 for the first long row, <= 1 per
    // long run (plus the rest of the first long row's run), + final flush.
    const size_t max_desc = 4 * static_cast<size_t>(R) + 16;
    Desc* desc = ctx->part_desc.as<Desc>(max_desc + 8);
    WalkOut* wout = reinterpret_cast<WalkOut*>(desc + max_desc);
    walk_kernel<<<1, kWalkThreads, 0, s>>>(p, d_rowoff, run_start, d_R, desc, wout);
    CWLB_LAUNCH_CHECK("walk_kernel");
    WalkOut w{};
    CWLB_CUDA(cudaMemcpyAsync(&w, wout, sizeof(w), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    if (w.fallback) return literal_partition(ctx, p, d_rowoff);
    if (w.n_tasks <= 0) return 0;

    cwlb_task* d_tasks = ctx->part_tasks.as<cwlb_task>(static_cast<size_t>(w.n_tasks));
    expand_kernel<<<static_cast<unsigned>(ceil_div(w.n_tasks, 256)), 256, 0, s>>>(p, desc, w.n_desc,
                                                                                  w.n_tasks, d_tasks);
    CWLB_LAUNCH_CHECK("expand_kernel");
    return w.n_tasks;
}

}  // namespace cwlb

// ===========================================================================
// No-allocation variant of the device partitioner.
//
// Some callers cannot let a library call cudaMalloc/cudaFree: their device
// memory belongs to another allocator (a framework's caching allocator, or a
// pool sized once at start-up by a server that must keep its footprint fixed),
// and cudaMalloc/cudaFree would also synchronise the device in the middle of
// their pipelines.  They can still pass input and output buffers.  For them,
// cwlb_partition_device_noalloc keeps all of its scratch in one file-scope
// device array of fixed size, g_noalloc_scratch below, which every GPU that
// loads this library holds until the process exits.  The array is shared by
// every call and keeps the previous call's contents; nothing in it has to
// start at zero (each piece is written before it is read).  Calls whose work
// overlaps on the GPU (two streams, two host threads) race on it and must be
// serialised by the caller.
// ===========================================================================

namespace cwlb {
namespace {

constexpr size_t kNoallocAlign = 256;
constexpr size_t noalloc_round(size_t b) { return (b + kNoallocAlign - 1) / kNoallocAlign * kNoallocAlign; }
constexpr size_t kNoallocPosBytes = noalloc_round(sizeof(int32_t) * CWLB_NOALLOC_MAX_ROWS);
constexpr size_t kNoallocScanBytes = 8192;  // scan tree for <= 2^20 items
constexpr size_t kNoallocRunBytes = noalloc_round(sizeof(int32_t) * (CWLB_NOALLOC_MAX_RUNS + 1));
constexpr size_t kNoallocMaxDesc = 4 * static_cast<size_t>(CWLB_NOALLOC_MAX_RUNS) + 16;
constexpr size_t kNoallocDescBytes = noalloc_round(sizeof(Desc) * kNoallocMaxDesc);
constexpr size_t kNoallocSmallBytes = 512;  // run count, walker summary, literal count
constexpr size_t kNoallocBytes =
    kNoallocPosBytes + kNoallocScanBytes + kNoallocRunBytes + kNoallocDescBytes + kNoallocSmallBytes;
static_assert(kNoallocBytes <= (8u << 20), "no-allocation scratch exceeds its stated 8 MiB");

// The scratch.  Host code must not use this name as a device address (in host
// code it is only a stand-in); it uses the address from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[8u << 20];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[256] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (the first call on each device; it must precede any stream
// capture that includes this entry point).
void* noalloc_scratch_current_device() {
    int dev = -1;
    CWLB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 256) fail(CWLB_ERR_RUNTIME, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        CWLB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        if (!p) fail(CWLB_ERR_CUDA, "cudaGetSymbolAddress returned a null address");
        g_noalloc_addr[dev] = p;
    }
    return g_noalloc_addr[dev];
}

// run_compact_kernel with a capacity: run starts beyond max_runs are not
// stored (the host then rejects the input); the run count is always stored.
__global__ void run_compact_capped_kernel(const int32_t* __restrict__ rowoff, int32_t n,
                                          const int32_t* __restrict__ pos, int32_t max_runs,
                                          int32_t* __restrict__ run_start,
                                          int32_t* __restrict__ n_runs) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t d = rowoff[i + 1] - rowoff[i];
    const bool start = (i == 0 || d != rowoff[i] - rowoff[i - 1]);
    if (start && pos[i] < max_runs) run_start[pos[i]] = static_cast<int32_t>(i);
    if (i == n - 1) {
        const int32_t r = pos[i] + (start ? 1 : 0);
        *n_runs = r;
        if (r <= max_runs) run_start[r] = n;
    }
}

int64_t partition_noalloc(cudaStream_t s, int32_t n_rows, const int32_t* d_rowoff,
                          const cwlb_costs& costs, double capacity, cwlb_task* d_tasks,
                          int64_t max_tasks) {
    if (n_rows > CWLB_NOALLOC_MAX_ROWS) {
        fail(CWLB_ERR_INVALID_ARGUMENT,
             "cwlb_partition_device_noalloc: " + std::to_string(n_rows) +
                 " rows exceed the no-allocation scratch limit of " +
                 std::to_string(CWLB_NOALLOC_MAX_ROWS) + " rows");
    }
    char* base = static_cast<char*>(noalloc_scratch_current_device());
    int32_t* pos = reinterpret_cast<int32_t*>(base);
    void* scan_tmp = base + kNoallocPosBytes;
    int32_t* run_start = reinterpret_cast<int32_t*>(base + kNoallocPosBytes + kNoallocScanBytes);
    Desc* desc = reinterpret_cast<Desc*>(base + kNoallocPosBytes + kNoallocScanBytes + kNoallocRunBytes);
    char* small = base + kNoallocPosBytes + kNoallocScanBytes + kNoallocRunBytes + kNoallocDescBytes;
    int32_t* d_R = reinterpret_cast<int32_t*>(small);
    WalkOut* wout = reinterpret_cast<WalkOut*>(small + 64);
    int64_t* d_count = reinterpret_cast<int64_t*>(small + 256);

    const Params p = make_params(n_rows, costs, capacity);
    const bool fast = std::isfinite(p.wCL) && std::isfinite(p.Cs) && std::isfinite(p.Ca) &&
                      std::isfinite(p.cap) && p.wCL > 0.0;
    auto literal = [&]() -> int64_t {
        literal_partition_kernel<<<1, 32, 0, s>>>(p, d_rowoff, d_tasks, max_tasks, d_count);
        CWLB_LAUNCH_CHECK("literal_partition_kernel");
        int64_t cnt = 0;
        CWLB_CUDA(cudaMemcpyAsync(&cnt, d_count, sizeof(cnt), cudaMemcpyDeviceToHost, s));
        CWLB_CUDA(cudaStreamSynchronize(s));
        return cnt;
    };
    if (!fast) return literal();

    const int64_t n = n_rows;
    const unsigned blocks = static_cast<unsigned>(ceil_div(n, 256));
    if (scan_scratch_bytes<int32_t>(n) > kNoallocScanBytes) fail(CWLB_ERR_RUNTIME, "scan scratch");
    run_flags_kernel<<<blocks, 256, 0, s>>>(d_rowoff, n_rows, pos);
    CWLB_LAUNCH_CHECK("run_flags_kernel");
    device_exclusive_scan<int32_t>(pos, pos, n, scan_tmp, s);
    run_compact_capped_kernel<<<blocks, 256, 0, s>>>(d_rowoff, n_rows, pos, CWLB_NOALLOC_MAX_RUNS,
                                                     run_start, d_R);
    CWLB_LAUNCH_CHECK("run_compact_capped_kernel");
    int32_t R = 0;
    CWLB_CUDA(cudaMemcpyAsync(&R, d_R, sizeof(R), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    if (R > CWLB_NOALLOC_MAX_RUNS) {
        fail(CWLB_ERR_INVALID_ARGUMENT,
             "cwlb_partition_device_noalloc: " + std::to_string(R) +
                 " distinct row degrees exceed the no-allocation scratch limit of " +
                 std::to_string(CWLB_NOALLOC_MAX_RUNS));
    }
    walk_kernel<<<1, kWalkThreads, 0, s>>>(p, d_rowoff, run_start, d_R, desc, wout);
    CWLB_LAUNCH_CHECK("walk_kernel");
    WalkOut w{};
    CWLB_CUDA(cudaMemcpyAsync(&w, wout, sizeof(w), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    if (w.fallback) return literal();
    if (w.n_tasks > max_tasks || w.n_tasks <= 0 || !d_tasks) return w.n_tasks;
    expand_kernel<<<static_cast<unsigned>(ceil_div(w.n_tasks, 256)), 256, 0, s>>>(p, desc, w.n_desc,
                                                                                  w.n_tasks, d_tasks);
    CWLB_LAUNCH_CHECK("expand_kernel");
    return w.n_tasks;
}

}  // namespace
}  // namespace cwlb

extern "C" int cwlb_partition_device_noalloc(void* cuda_stream, int32_t n_rows,
                                             const int32_t* d_row_offset, const cwlb_costs* costs,
                                             double capacity, cwlb_task* d_tasks,
                                             int64_t max_tasks, int64_t* n_tasks) {
    try {
        // Checked before any launch: a NULL task buffer with a positive
        // capacity would otherwise reach the expansion kernel's stores.
        if (!costs || !n_tasks || (n_rows > 0 && !d_row_offset) || max_tasks < 0 ||
            (max_tasks > 0 && !d_tasks)) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "cwlb_partition_device_noalloc: null argument");
        }
        *n_tasks = 0;
        if (n_rows <= 0) return CWLB_OK;
        const int64_t cnt = cwlb::partition_noalloc(static_cast<cudaStream_t>(cuda_stream), n_rows,
                                                    d_row_offset, *costs, capacity, d_tasks,
                                                    max_tasks);
        *n_tasks = cnt;
        if (cnt > max_tasks) {
            cwlb::fail(CWLB_ERR_BUFFER_TOO_SMALL,
                       "cwlb_partition_device_noalloc: the task buffer holds " +
                           std::to_string(max_tasks) + " tasks, " + std::to_string(cnt) +
                           " are needed");
        }
        return CWLB_OK;
    } catch (const cwlb::Failure& e) {
        cwlb::set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        cwlb::set_last_error(e.what());
        return CWLB_ERR_RUNTIME;
    }
}
