// Aggregation plans: the task list of a reordered CSR prepared once for many
// launches (the reference's 70-launch timing loop, main.cpp:372-406, or one
// graph layer after another).
//
// Where the time goes without a plan: every nonzero gathers one row of H
// (4K bytes) from L2, and on power-law graphs most nonzeros sit in hub rows
// that the partitioner (src/utils.cpp:985-1010) cuts into single-row
// fragment tasks of about S nonzeros.  Fragments of hub rows with similar
// degree at similar positions reference many of the same columns (the hub
// columns): on the R-MAT configuration 2 graph, 8 such fragments reference
// about 0.6 distinct columns per nonzero.
//
// A plan therefore GROUPS single-row fragment tasks, R = 4 (or 8) per group,
// taken from blocks of kRowBlock consecutive rows in order of their first
// column, and stores each group's merged union of nonzeros bucketed by the
// MASK of members holding each column: runs of equal mask, columns ascending
// inside a run.  One warp then runs a whole group: each distinct column's H
// row is loaded once, a run's rows are summed in registers, and the run's sum
// is added to the register accumulator of each member in its mask; each
// member is finally divided by its row's full degree and added atomically to
// the output row, exactly as the task kernel writes a fragment.  Every task
// still covers exactly its own nonzeros; only the order of additions inside a
// fragment changes (runs, then columns), which the tolerance covers, as it
// covers the atomic merge of fragments.  Tasks that cover a whole row are not
// grouped, so whole rows are computed exactly as without a plan.  Tasks that
// are not grouped (several rows, a whole row, empty, or longer than
// kMaxMemberNnz) run through the task kernel with a launch order.
//
// Groups are used only when the plan can show they are exact and pay:
// every grouped nonzero has value 1.0f (the adds need no multiply; the
// reference's loader gives every stored entry the value 1, src/data.cpp:115),
// every grouped fragment's columns are non-decreasing, and the union is at
// most kMaxUnionRatio of the grouped nonzeros.  Otherwise the plan runs the
// task kernel over all tasks, unchanged.
#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "scan.cuh"

struct cwlb_plan {
    cwlb_ctx* ctx = nullptr;
    int32_t n_rows = 0, nnz = 0;
    const int32_t* rowoff = nullptr;
    const int32_t* col = nullptr;
    const float* val = nullptr;
    const cwlb_task* tasks = nullptr;
    int64_t n_tasks = 0;
    int32_t R = 0;             // members per group; 0 = no groups
    int64_t n_groups = 0, n_rest = 0, grouped_tasks = 0, grouped_nnz = 0, union_entries = 0;
    uint32_t off_reason = 0;   // CWLB_PLAN_* bits: why groups are not used
    cwlb::DeviceBuffer gtask, goff, gcount, ucol, runs, nruns, rest;
};

namespace cwlb {
namespace {

constexpr int kPlanThreads = 256;
constexpr int kRowBlock = 64;          // rows whose fragments may share a group
constexpr int32_t kMaxMemberNnz = 4096;
constexpr double kMaxUnionRatio = 0.75;  // configuration 5 (0.81) measured slower with groups
constexpr int32_t kEnd = 0x7fffffff;   // merge: member exhausted

// Build-time status bits (device word, read once by the host).
constexpr uint32_t kBadValue = 1u;     // a grouped nonzero is not 1.0f
constexpr uint32_t kUnsorted = 2u;     // a grouped fragment's columns decrease

struct BuildStats {
    unsigned long long union_entries;
    unsigned int flags;
    unsigned int max_col;
    unsigned int max_block;
    unsigned int pad;
};

struct Frag {
    int32_t base, begin, end, deg;
};

// Task t's single-row fragment, or false when t is not a single row with a
// non-empty fragment (the clamping of row_fragment in spmm.cu).
__device__ __forceinline__ bool single_fragment(const int32_t* __restrict__ rowoff, int32_t n_rows,
                                                int32_t nnz, const cwlb_task& tk, Frag& f) {
    if (tk.row_start < 0 || tk.row_end > n_rows || tk.row_end != tk.row_start + 1) return false;
    const int32_t r = tk.row_start;
    const int32_t b0 = rowoff[r], b1 = rowoff[r + 1];
    if (b0 < 0 || b1 < b0 || b1 > nnz) return false;
    const int32_t deg = b1 - b0;
    if (deg <= 0) return false;
    int32_t begin = tk.first_row_offset;
    int32_t end = tk.last_row_nnz > 0 ? tk.last_row_nnz : deg;
    begin = min(max(begin, 0), deg);
    end = min(max(end, begin), deg);
    f = Frag{b0, begin, end, deg};
    return begin < end;
}

__global__ void plan_classify_kernel(const int32_t* __restrict__ rowoff, int32_t n_rows,
                                     int32_t nnz, const int32_t* __restrict__ col,
                                     const cwlb_task* __restrict__ tasks, int64_t n_tasks,
                                     int32_t* __restrict__ is_cand, int32_t* __restrict__ fnnz,
                                     BuildStats* __restrict__ st) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    unsigned mc = 0, mb = 0;
    if (t < n_tasks) {
        const cwlb_task tk = tasks[t];
        Frag f;
        // Fragments only: a task that covers a whole row stays with the task
        // kernel.
        const bool c = single_fragment(rowoff, n_rows, nnz, tk, f) &&
                       f.end - f.begin <= kMaxMemberNnz && !(f.begin == 0 && f.end == f.deg);
        is_cand[t] = c ? 1 : 0;
        fnnz[t] = c ? f.end - f.begin : 0;
        if (c) {
            mc = static_cast<unsigned>(max(col[f.base + f.begin], 0));
            mb = static_cast<unsigned>(tk.row_start / kRowBlock);
        }
    }
    mc = __reduce_max_sync(0xffffffffu, mc);
    mb = __reduce_max_sync(0xffffffffu, mb);
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&st->max_col, mc);
        atomicMax(&st->max_block, mb);
    }
}

// Candidates in task order (keys: first column, row block; value: position)
// and the other tasks in task order.
__global__ void plan_compact_kernel(const int32_t* __restrict__ rowoff, int32_t n_rows,
                                    int32_t nnz, const int32_t* __restrict__ col,
                                    const cwlb_task* __restrict__ tasks, int64_t n_tasks,
                                    const int32_t* __restrict__ is_cand,
                                    const int32_t* __restrict__ pos,
                                    int32_t* __restrict__ cand_task, uint32_t* __restrict__ key_col,
                                    uint32_t* __restrict__ key_blk, int32_t* __restrict__ idx,
                                    int32_t* __restrict__ rest) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n_tasks) return;
    const int32_t p = pos[t];
    if (is_cand[t]) {
        const cwlb_task tk = tasks[t];
        Frag f{0, 0, 0, 0};
        single_fragment(rowoff, n_rows, nnz, tk, f);  // true: classified as a candidate
        cand_task[p] = static_cast<int32_t>(t);
        key_col[p] = static_cast<uint32_t>(max(col[f.base + f.begin], 0));
        key_blk[p] = static_cast<uint32_t>(tk.row_start / kRowBlock);
        idx[p] = p;
    } else {
        rest[t - p] = static_cast<int32_t>(t);
    }
}

__global__ void plan_gather_keys_kernel(const uint32_t* __restrict__ key_blk,
                                        const int32_t* __restrict__ idx, int32_t n,
                                        uint32_t* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = key_blk[idx[i]];
}

// Group g = sorted candidates [g R, g R + R): member task ids (-1 = none)
// and an upper bound of the union length (the members' nonzeros).
__global__ void plan_groups_kernel(const int32_t* __restrict__ cand_task,
                                   const int32_t* __restrict__ idx, int32_t n_cand, int R,
                                   int64_t n_groups, const int32_t* __restrict__ fnnz,
                                   int32_t* __restrict__ gtask, int32_t* __restrict__ gbound) {
    const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (g >= n_groups) return;
    int32_t bound = 0;
    for (int m = 0; m < R; ++m) {
        const int64_t i = g * R + m;
        int32_t t = -1;
        if (i < n_cand) {
            t = cand_task[idx[i]];
            bound += fnnz[t];
        }
        gtask[g * R + m] = t;
    }
    gbound[g] = bound;
}

// Merge state of one member (lane m walks member m's column-sorted fragment).
struct Merge {
    int32_t pos, end, cur, nxt;
};

__device__ __forceinline__ void merge_start(const int32_t* __restrict__ rowoff, int32_t n_rows,
                                            int32_t nnz, const int32_t* __restrict__ col,
                                            const cwlb_task* __restrict__ tasks,
                                            const int32_t* __restrict__ gtask, int64_t g, int R,
                                            int lane, Merge& m) {
    m = Merge{0, 0, kEnd, kEnd};
    if (lane < R) {
        const int32_t t = gtask[g * R + lane];
        Frag f;
        if (t >= 0 && single_fragment(rowoff, n_rows, nnz, tasks[t], f)) {
            m.pos = f.base + f.begin;
            m.end = f.base + f.end;
            m.cur = col[m.pos];
            m.nxt = m.pos + 1 < m.end ? col[m.pos + 1] : kEnd;
        }
    }
}

// The next union entry (column, mask of the members holding it), or false
// when every member is exhausted.  All lanes of the warp call it together.
__device__ __forceinline__ bool merge_next(const int32_t* __restrict__ col, Merge& m,
                                           int32_t& c_out, unsigned& mask_out) {
    int32_t c = m.cur;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c = min(c, __shfl_xor_sync(0xffffffffu, c, o));
    if (c == kEnd) return false;
    const bool take = m.cur == c;
    mask_out = __ballot_sync(0xffffffffu, take);
    c_out = c;
    if (take) {
        ++m.pos;
        if (m.pos < m.end) {
            m.cur = m.nxt;
            m.nxt = m.pos + 1 < m.end ? col[m.pos + 1] : kEnd;
        } else {
            m.cur = kEnd;
        }
    }
    return true;
}

// One warp per group.  Pass 1 counts the union's entries per member mask in a
// per-warp histogram and writes the group's RUN table (one word per mask
// present, in ascending mask order: mask << 24 | entries); pass 2 merges
// again and writes each entry's column into its mask's run, so that the
// columns of a run are ascending.  gcount[g] = entries written.  Pass 1 also
// checks that the values are 1.0f and the columns do not decrease.
template <int R>
__global__ void __launch_bounds__(kPlanThreads)
    plan_merge_kernel(const int32_t* __restrict__ rowoff, int32_t n_rows, int32_t nnz,
                      const int32_t* __restrict__ col, const float* __restrict__ val,
                      const cwlb_task* __restrict__ tasks, int64_t n_groups,
                      const int32_t* __restrict__ gtask, const int32_t* __restrict__ goff,
                      int32_t* __restrict__ gcount, int32_t* __restrict__ nruns,
                      uint32_t* __restrict__ runs, int32_t* __restrict__ ucol,
                      BuildStats* __restrict__ st) {
    constexpr int kBins = 1 << R;
    constexpr int kPer = (kBins + 31) / 32;  // bins per lane
    __shared__ int32_t hist_all[kPlanThreads / 32][kBins];
    const int lane = threadIdx.x & 31;
    int32_t* hist = hist_all[threadIdx.x >> 5];
    const int64_t g = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (g >= n_groups) return;
    for (int b = lane; b < kBins; b += 32) hist[b] = 0;
    __syncwarp();

    // Pass 1: count entries per mask; check values and order.
    Merge m;
    merge_start(rowoff, n_rows, nnz, col, tasks, gtask, g, R, lane, m);
    uint32_t bad = 0;
    if (m.pos < m.end) {
        if (val && val[m.pos] != 1.0f) bad |= kBadValue;
        // A stored column equal to the end marker (never a valid index of H)
        // would end this member early: refuse to group instead.
        if (m.cur == kEnd || (m.pos + 1 < m.end && m.nxt == kEnd)) bad |= kUnsorted;
    }
    const int32_t base = goff[g];
    const int32_t cap = goff[g + 1] - base;
    int32_t k = 0;
    for (;;) {
        const int32_t prev_cur = m.cur;
        const int32_t prev_pos = m.pos;
        int32_t c;
        unsigned mask;
        if (!merge_next(col, m, c, mask)) break;
        if (lane == 0) hist[mask & (kBins - 1)] += 1;
        ++k;
        if (m.pos != prev_pos && m.pos < m.end) {
            if (m.cur < prev_cur) bad |= kUnsorted;
            if (val && val[m.pos] != 1.0f) bad |= kBadValue;
            if (m.pos + 1 < m.end && m.nxt == kEnd) bad |= kUnsorted;
        }
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    __syncwarp();
    // Runs: bins in ascending mask order, lane l holding bins [l kPer, l kPer + kPer).
    int32_t cnt[kPer], nonzero = 0, total = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const int b = lane * kPer + q;
        cnt[q] = b < kBins ? hist[b] : 0;
        total += cnt[q];
        nonzero += cnt[q] > 0;
    }
    int32_t off = total, rix = nonzero;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int32_t a = __shfl_up_sync(0xffffffffu, off, o);
        const int32_t r = __shfl_up_sync(0xffffffffu, rix, o);
        if (lane >= o) {
            off += a;
            rix += r;
        }
    }
    off -= total;  // exclusive
    rix -= nonzero;
    __syncwarp();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const int b = lane * kPer + q;
        if (b < kBins) hist[b] = off;  // first slot of bin b's run
        if (cnt[q] > 0) {
            runs[g * kBins + rix] = (static_cast<uint32_t>(b) << 24) | static_cast<uint32_t>(cnt[q]);
            ++rix;
        }
        off += cnt[q];
    }
    const int32_t n_runs = __shfl_sync(0xffffffffu, rix, 31);
    __syncwarp();

    // Pass 2: write each entry's column into its run.
    merge_start(rowoff, n_rows, nnz, col, tasks, gtask, g, R, lane, m);
    for (;;) {
        int32_t c;
        unsigned mask;
        if (!merge_next(col, m, c, mask)) break;
        if (lane == 0) {
            const int32_t slot = hist[mask & (kBins - 1)]++;
            if (slot < cap) ucol[base + slot] = c;
        }
    }
    if (lane == 0) {
        gcount[g] = min(k, cap);
        nruns[g] = n_runs;
        atomicAdd(&st->union_entries, static_cast<unsigned long long>(k));
        if (bad) atomicOr(&st->flags, bad);
    }
}

// ---------------------------------------------------------------------------
// The group kernel.

#ifndef CWLB_GROUP_MIN_BLOCKS
#define CWLB_GROUP_MIN_BLOCKS 2
#endif
constexpr int kGroupMinBlocks = CWLB_GROUP_MIN_BLOCKS;  // CTAs per SM the registers allow

template <int VW>
struct VecT;
template <>
struct VecT<1> {
    using T = float;
    // Loads are volatile so that they are issued where written (all of a
    // step's loads before its adds) and not sunk into the member dispatch.
    __device__ static T load(const T* p) {
        T v;
        asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
        return v;
    }
    __device__ static T zero() { return 0.0f; }
    __device__ static void add(T& a, const T& x) { a += x; }
    __device__ static T div(const T& a, float d) { return __fdiv_rn(a, d); }
};
template <>
struct VecT<2> {
    using T = float2;
    __device__ static T load(const T* p) {
        T v;
        asm volatile("ld.global.nc.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
        return v;
    }
    __device__ static T zero() { return make_float2(0.f, 0.f); }
    __device__ static void add(T& a, const T& x) {
        a.x += x.x;
        a.y += x.y;
    }
    __device__ static T div(const T& a, float d) { return make_float2(__fdiv_rn(a.x, d), __fdiv_rn(a.y, d)); }
};
template <>
struct VecT<4> {
    using T = float4;
    __device__ static T load(const T* p) {
        T v;
        asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                     : "l"(p));
        return v;
    }
    __device__ static T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
    __device__ static void add(T& a, const T& x) {
        a.x += x.x;
        a.y += x.y;
        a.z += x.z;
        a.w += x.w;
    }
    __device__ static T div(const T& a, float d) {
        return make_float4(__fdiv_rn(a.x, d), __fdiv_rn(a.y, d), __fdiv_rn(a.z, d), __fdiv_rn(a.w, d));
    }
};

struct GroupArgs {
    const int32_t* __restrict__ rowoff;
    const int32_t* __restrict__ origin;
    const cwlb_task* __restrict__ tasks;
    const int32_t* __restrict__ gtask;
    const int32_t* __restrict__ goff;
    const int32_t* __restrict__ gcount;
    const int32_t* __restrict__ nruns;
    const uint32_t* __restrict__ runs;
    const int32_t* __restrict__ ucol;
    const float* __restrict__ H;
    float* __restrict__ out;
    uint32_t* err;
    int64_t h_rows;
    int64_t n_groups;
    int32_t n_rows;
    int32_t nnz;
};

// acc[b] += x for a warp-uniform member index b (a jump table keeps the
// accumulators in registers).
template <int R, typename V, typename T>
__device__ __forceinline__ void add_member(T (&acc)[R], int b, const T& x) {
    switch (b) {
#define CWLB_MEMBER_CASE(i) \
    case i:                 \
        if constexpr (i < R) V::add(acc[i], x); \
        break;
        CWLB_MEMBER_CASE(0) CWLB_MEMBER_CASE(1) CWLB_MEMBER_CASE(2) CWLB_MEMBER_CASE(3)
        CWLB_MEMBER_CASE(4) CWLB_MEMBER_CASE(5) CWLB_MEMBER_CASE(6) CWLB_MEMBER_CASE(7)
#undef CWLB_MEMBER_CASE
        default: break;
    }
}

// One warp per group, VW floats of each H row per lane (K = 32 VW), U loads in
// flight.  The group's entries come as runs of equal member mask: a run's H
// rows are summed into s, and s is added to each of the run's members once.
template <int VW, int R, int U>
__global__ void __launch_bounds__(kPlanThreads, kGroupMinBlocks) group_kernel(GroupArgs a) {
    using V = VecT<VW>;
    using T = typename V::T;
    constexpr int kBins = 1 << R;
    const int lane = threadIdx.x & 31;
    // Groups run heaviest first: they are stored in ascending row (degree)
    // order, and the hub groups at the end hold the most entries.
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (w >= a.n_groups) return;
    const int64_t g = a.n_groups - 1 - w;

    // Lane m < R describes member m (its row's origin and degree).
    int32_t m_orig = 0;
    float m_deg = 1.0f;
    int m_ok = 0;
    if (lane < R) {
        const int32_t t = __ldg(a.gtask + g * R + lane);
        if (t >= 0) {
            const cwlb_task tk = a.tasks[t];
            Frag f;
            if (single_fragment(a.rowoff, a.n_rows, a.nnz, tk, f)) {
                const int32_t o = __ldg(a.origin + tk.row_start);
                if (o >= 0 && o < a.n_rows) {
                    m_orig = o;
                    m_deg = static_cast<float>(f.deg);
                    m_ok = 1;
                } else {
                    atomicOr(a.err, CWLB_DEVERR_ORIGIN_RANGE);
                }
            }
        }
    }

    T acc[R];
#pragma unroll
    for (int b = 0; b < R; ++b) acc[b] = V::zero();
    const T* __restrict__ Hv = reinterpret_cast<const T*>(a.H);
    const int32_t e0 = __ldg(a.goff + g);
    const int32_t ne = __ldg(a.gcount + g);
    const int32_t nr = __ldg(a.nruns + g);
    const uint32_t* __restrict__ runs = a.runs + g * kBins;
    // Run cursor: lane i holds run word (ri & ~31) + i.
    int32_t ri = 0;
    uint32_t run_chunk = lane < nr ? __ldg(runs + lane) : 0u;
    uint32_t rw = __shfl_sync(0xffffffffu, run_chunk, 0);
    int32_t run_left = static_cast<int32_t>(rw & 0xffffffu);
    T s = V::zero();
    for (int32_t c0 = 0; c0 < ne; c0 += 32) {
        const int32_t cnt = min(32, ne - c0);
        // Column of this lane's entry; bit 31 marks a column outside H
        // (flagged, read as row 0 and not added).
        uint32_t my_col = 0;
        if (lane < cnt) {
            const int32_t c = __ldg(a.ucol + e0 + c0 + lane);
            if (static_cast<uint32_t>(c) >= static_cast<uint64_t>(a.h_rows)) {
                atomicOr(a.err, CWLB_DEVERR_COL_RANGE);
                my_col = 0x80000000u;
            } else {
                my_col = static_cast<uint32_t>(c);
            }
        }
        const bool chunk_ok = !__any_sync(0xffffffffu, my_col >> 31);
        for (int32_t j = 0; j < cnt; j += U) {
            uint32_t cj[U];
            T x[U];
#pragma unroll
            for (int u = 0; u < U; ++u) cj[u] = __shfl_sync(0xffffffffu, my_col, (j + u) & 31);
#pragma unroll
            for (int u = 0; u < U; ++u)
                x[u] = V::load(Hv + static_cast<size_t>(cj[u] & 0x7fffffffu) * 32 + lane);
            if (chunk_ok && j + U <= cnt && run_left > U) {
                // The whole step lies inside the current run: sum it as a
                // tree (short dependency chains) and skip the bookkeeping.
#pragma unroll
                for (int w = 1; w < U; w <<= 1) {
#pragma unroll
                    for (int u = 0; u + w < U; u += 2 * w) V::add(x[u], x[u + w]);
                }
                V::add(s, x[0]);
                run_left -= U;
                continue;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (j + u >= cnt) break;
                if (!(cj[u] >> 31)) V::add(s, x[u]);
                if (--run_left == 0) {
                    // End of the run: add its sum to each member of its mask.
                    uint32_t mask = (rw >> 24) & (kBins - 1);
                    while (mask) {
                        const int b = __ffs(mask) - 1;
                        mask &= mask - 1;
                        add_member<R, V>(acc, b, s);
                    }
                    s = V::zero();
                    ++ri;
                    if (ri < nr) {
                        if ((ri & 31) == 0)
                            run_chunk = ri + lane < nr ? __ldg(runs + ri + lane) : 0u;
                        rw = __shfl_sync(0xffffffffu, run_chunk, ri & 31);
                        run_left = static_cast<int32_t>(rw & 0xffffffu);
                    }
                }
            }
        }
    }

#pragma unroll
    for (int b = 0; b < R; ++b) {
        const int ok = __shfl_sync(0xffffffffu, m_ok, b);
        if (!ok) continue;
        const int32_t o = __shfl_sync(0xffffffffu, m_orig, b);
        const float d = __shfl_sync(0xffffffffu, m_deg, b);
        T* dst = reinterpret_cast<T*>(a.out + static_cast<int64_t>(o) * (32 * VW)) + lane;
        atomicAdd(dst, V::div(acc[b], d));  // members are fragments: always added
    }
}

template <int VW, int R>
void launch_group(const GroupArgs& a, cudaStream_t s) {
    const unsigned grid = static_cast<unsigned>(ceil_div(a.n_groups, kPlanThreads / 32));
    group_kernel<VW, R, 4><<<grid, kPlanThreads, 0, s>>>(a);
    CWLB_LAUNCH_CHECK("group_kernel");
}

template <int VW>
void launch_group_r(int R, const GroupArgs& a, cudaStream_t s) {
    if (R <= 4) launch_group<VW, 4>(a, s);
    else launch_group<VW, 8>(a, s);
}

int bits_for(uint32_t v) {
    int b = 0;
    while (b < 32 && (v >> b) != 0u) ++b;
    return b;
}

void build_plan(cwlb_plan* p, int32_t group_size) {
    cwlb_ctx* ctx = p->ctx;
    cudaStream_t s = ctx->stream;
    const int64_t n = p->n_tasks;
    auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    // Per-task scratch: candidate flag, fragment nnz, positions, scan tree.
    const size_t b_t = al(sizeof(int32_t) * static_cast<size_t>(n));
    const size_t b_scan = al(scan_scratch_bytes<int32_t>(n));
    DeviceBuffer tmp;
    char* base = static_cast<char*>(tmp.ensure(3 * b_t + b_scan + al(sizeof(BuildStats))));
    int32_t* is_cand = reinterpret_cast<int32_t*>(base);
    int32_t* fnnz = reinterpret_cast<int32_t*>(base + b_t);
    int32_t* pos = reinterpret_cast<int32_t*>(base + 2 * b_t);
    void* scan_tmp = base + 3 * b_t;
    BuildStats* st = reinterpret_cast<BuildStats*>(base + 3 * b_t + b_scan);
    CWLB_CUDA(cudaMemsetAsync(st, 0, sizeof(BuildStats), s));
    const unsigned tb = static_cast<unsigned>(ceil_div(n, kPlanThreads));
    plan_classify_kernel<<<tb, kPlanThreads, 0, s>>>(p->rowoff, p->n_rows, p->nnz, p->col, p->tasks,
                                                      n, is_cand, fnnz, st);
    CWLB_LAUNCH_CHECK("plan_classify_kernel");
    device_exclusive_scan<int32_t>(is_cand, pos, n, scan_tmp, s);
    int32_t last_pos = 0, last_flag = 0;
    BuildStats hs{};
    CWLB_CUDA(cudaMemcpyAsync(&last_pos, pos + n - 1, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaMemcpyAsync(&last_flag, is_cand + n - 1, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaMemcpyAsync(&hs, st, sizeof(hs), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    const int32_t n_cand = last_pos + last_flag;
    const int64_t R = group_size;
    if (n_cand < 2 * R) {
        p->off_reason |= CWLB_PLAN_FEW_FRAGMENTS;
        return;
    }
    // Candidates sorted by (row block, first column), stable.
    const size_t b_c = al(sizeof(int32_t) * static_cast<size_t>(n_cand));
    DeviceBuffer ctmp;
    const size_t sort_b = radix_sort_pairs_scratch_bytes(n_cand, ctx->props.multiProcessorCount);
    char* cb = static_cast<char*>(ctmp.ensure(4 * b_c + sort_b));
    int32_t* cand_task = reinterpret_cast<int32_t*>(cb);
    uint32_t* key_col = reinterpret_cast<uint32_t*>(cb + b_c);
    uint32_t* key_blk = reinterpret_cast<uint32_t*>(cb + 2 * b_c);
    int32_t* idx = reinterpret_cast<int32_t*>(cb + 3 * b_c);
    void* sort_tmp = cb + 4 * b_c;
    p->n_rest = n - n_cand;
    int32_t* rest = p->rest.as<int32_t>(static_cast<size_t>(std::max<int64_t>(p->n_rest, 1)));
    plan_compact_kernel<<<tb, kPlanThreads, 0, s>>>(p->rowoff, p->n_rows, p->nnz, p->col, p->tasks,
                                                     n, is_cand, pos, cand_task, key_col, key_blk,
                                                     idx, rest);
    CWLB_LAUNCH_CHECK("plan_compact_kernel");
    radix_sort_pairs(ctx, key_col, idx, n_cand, bits_for(hs.max_col), sort_tmp);
    plan_gather_keys_kernel<<<static_cast<unsigned>(ceil_div(n_cand, kPlanThreads)), kPlanThreads, 0,
                              s>>>(key_blk, idx, n_cand, key_col);
    CWLB_LAUNCH_CHECK("plan_gather_keys_kernel");
    radix_sort_pairs(ctx, key_col, idx, n_cand, bits_for(hs.max_block), sort_tmp);

    const int64_t n_groups = ceil_div(n_cand, R);
    int32_t* gtask = p->gtask.as<int32_t>(static_cast<size_t>(n_groups * R));
    int32_t* goff = p->goff.as<int32_t>(static_cast<size_t>(n_groups) + 1);
    int32_t* gcount = p->gcount.as<int32_t>(static_cast<size_t>(n_groups));
    // goff = exclusive scan of the union bounds, with a trailing total.
    DeviceBuffer gscan;
    int32_t* gb = gscan.as<int32_t>(static_cast<size_t>(n_groups) + 1);
    plan_groups_kernel<<<static_cast<unsigned>(ceil_div(n_groups, kPlanThreads)), kPlanThreads, 0,
                         s>>>(cand_task, idx, n_cand, static_cast<int>(R), n_groups, fnnz, gtask,
                              gb);
    CWLB_LAUNCH_CHECK("plan_groups_kernel");
    CWLB_CUDA(cudaMemsetAsync(gb + n_groups, 0, sizeof(int32_t), s));
    DeviceBuffer gscan_tmp;
    device_exclusive_scan<int32_t>(gb, goff, n_groups + 1,
                                   gscan_tmp.ensure(scan_scratch_bytes<int32_t>(n_groups + 1)), s);
    int32_t bound_total = 0;
    CWLB_CUDA(cudaMemcpyAsync(&bound_total, goff + n_groups, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    int32_t* ucol = p->ucol.as<int32_t>(static_cast<size_t>(std::max(bound_total, 1)));
    const int64_t bins = int64_t{1} << R;
    uint32_t* runs = p->runs.as<uint32_t>(static_cast<size_t>(n_groups * bins));
    int32_t* nruns = p->nruns.as<int32_t>(static_cast<size_t>(n_groups));
    const unsigned mg = static_cast<unsigned>(ceil_div(n_groups * 32, kPlanThreads));
    if (R <= 4) {
        plan_merge_kernel<4><<<mg, kPlanThreads, 0, s>>>(p->rowoff, p->n_rows, p->nnz, p->col,
                                                         p->val, p->tasks, n_groups, gtask, goff,
                                                         gcount, nruns, runs, ucol, st);
    } else {
        plan_merge_kernel<8><<<mg, kPlanThreads, 0, s>>>(p->rowoff, p->n_rows, p->nnz, p->col,
                                                         p->val, p->tasks, n_groups, gtask, goff,
                                                         gcount, nruns, runs, ucol, st);
    }
    CWLB_LAUNCH_CHECK("plan_merge_kernel");
    CWLB_CUDA(cudaMemcpyAsync(&hs, st, sizeof(hs), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    p->grouped_tasks = n_cand;
    p->grouped_nnz = bound_total;
    p->union_entries = static_cast<int64_t>(hs.union_entries);
    if (hs.flags & kBadValue) p->off_reason |= CWLB_PLAN_VALUES;
    if (hs.flags & kUnsorted) p->off_reason |= CWLB_PLAN_UNSORTED;
    if (static_cast<double>(p->union_entries) > kMaxUnionRatio * static_cast<double>(bound_total))
        p->off_reason |= CWLB_PLAN_NO_REUSE;
    if (p->off_reason) return;
    p->R = static_cast<int32_t>(R);
    p->n_groups = n_groups;
}

void release_groups(cwlb_plan* p) {
    for (DeviceBuffer* b : {&p->gtask, &p->goff, &p->gcount, &p->ucol, &p->runs, &p->nruns, &p->rest})
        b->release();
    p->R = 0;
    p->n_groups = 0;
    p->n_rest = p->n_tasks;
}

}  // namespace

void plan_aggregate(cwlb_plan* p, const int32_t* origin, const float* H, int64_t h_rows, int64_t K,
                    float* out, uint32_t flags) {
    cwlb_ctx* ctx = p->ctx;
    const bool aligned = (reinterpret_cast<uintptr_t>(H) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    const bool groups = p->n_groups > 0 && aligned && (K == 32 || K == 64 || K == 128) &&
                        !(flags & CWLB_DETERMINISTIC) && p->n_rows > 0;
    if (!groups) {
        launch_spmm_mean(ctx, p->n_rows, p->nnz, p->rowoff, p->col, p->val, origin, H, h_rows, K,
                         p->tasks, p->n_tasks, out, flags);
        return;
    }
    if (p->nnz > 0 && h_rows <= 0) fail(CWLB_ERR_INVALID_ARGUMENT, "H has no rows but the CSR has nonzeros");
    // 1. The zero-fill (or the split-row zeroing) over all tasks.
    // 2. The ungrouped tasks on the context's stream and the groups on its
    //    second stream, concurrently: rows that a task covers whole, and
    //    empty rows, are written only by ungrouped tasks; rows split between
    //    tasks only receive atomic adds after step 1.
    // 3. The context's stream waits for the groups.
    const int32_t* rest = p->rest.as<int32_t>(1);
    launch_spmm_mean(ctx, p->n_rows, p->nnz, p->rowoff, p->col, p->val, origin, H, h_rows, K,
                     p->tasks, p->n_tasks, out, flags, rest, 0);
    CWLB_CUDA(cudaEventRecord(ctx->plan_fork, ctx->stream));
    CWLB_CUDA(cudaStreamWaitEvent(ctx->copy_stream, ctx->plan_fork, 0));
    // The ungrouped tasks run in the variant the whole list would (their
    // rows then equal the task kernel's bit for bit).
    launch_spmm_mean(ctx, p->n_rows, p->nnz, p->rowoff, p->col, p->val, origin, H, h_rows, K,
                     p->tasks, p->n_tasks, out,
                     flags | kFlagOutCleared | kFlagSplitZeroed |
                         task_variant_flag(ctx, p->n_tasks, flags),
                     rest, p->n_rest);
    GroupArgs a{};
    a.rowoff = p->rowoff;
    a.origin = origin;
    a.tasks = p->tasks;
    a.gtask = p->gtask.as<int32_t>(1);
    a.goff = p->goff.as<int32_t>(1);
    a.gcount = p->gcount.as<int32_t>(1);
    a.nruns = p->nruns.as<int32_t>(1);
    a.runs = p->runs.as<uint32_t>(1);
    a.ucol = p->ucol.as<int32_t>(1);
    a.H = H;
    a.out = out;
    a.err = ctx->d_error_flags;
    a.h_rows = h_rows;
    a.n_groups = p->n_groups;
    a.n_rows = p->n_rows;
    a.nnz = p->nnz;
    switch (K) {
        case 32: launch_group_r<1>(p->R, a, ctx->copy_stream); break;
        case 64: launch_group_r<2>(p->R, a, ctx->copy_stream); break;
        default: launch_group_r<4>(p->R, a, ctx->copy_stream); break;
    }
    CWLB_CUDA(cudaEventRecord(ctx->plan_join, ctx->copy_stream));
    CWLB_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->plan_join, 0));
}

cwlb_plan* plan_create(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                       const int32_t* col, const float* val, const cwlb_task* tasks,
                       int64_t n_tasks, int32_t group_size) {
    if (group_size > 8) fail(CWLB_ERR_INVALID_ARGUMENT, "group_size must be at most 8");
    auto* p = new cwlb_plan();
    p->ctx = ctx;
    p->n_rows = n_rows;
    p->nnz = nnz;
    p->rowoff = rowoff;
    p->col = col;
    p->val = val;
    p->tasks = tasks;
    p->n_tasks = n_tasks;
    p->n_rest = n_tasks;
    try {
        // Values that are all 1.0 are not read at all (the task kernel's
        // unit-value instances); the plan then keeps no value pointer.
        if (nnz > 0) {
            DeviceBuffer flag;
            if (values_all_one(ctx, val, static_cast<size_t>(nnz),
                               static_cast<unsigned int*>(flag.ensure(sizeof(unsigned int)))))
                p->val = nullptr;
        }
        if (group_size == 0) group_size = 4;  // measured faster than 8 on B200
        if (group_size <= 1) {
            p->off_reason |= CWLB_PLAN_DISABLED;
        } else {
            group_size = group_size <= 4 ? 4 : 8;  // the kernels' two sizes
            if (n_rows > 0 && n_tasks > 0 && nnz > 0) build_plan(p, group_size);
        }
        if (p->n_groups == 0) release_groups(p);
    } catch (...) {
        release_groups(p);
        delete p;
        throw;
    }
    return p;
}

void plan_destroy(cwlb_plan* p) {
    if (!p) return;
    if (p->ctx) cudaSetDevice(p->ctx->device);
    release_groups(p);
    delete p;
}

}  // namespace cwlb

extern "C" {

int cwlb_plan_create(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* d_row_offset,
                     const int32_t* d_col_ind, const float* d_value, const cwlb_task* d_tasks,
                     int64_t n_tasks, int32_t group_size, cwlb_plan** out) {
    try {
        if (!ctx || !out) cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "null argument");
        *out = nullptr;
        if (n_rows < 0 || nnz < 0 || n_tasks < 0 || group_size < 0) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "negative size");
        }
        if ((n_rows > 0 && !d_row_offset) || (nnz > 0 && (!d_col_ind || !d_value)) ||
            (n_tasks > 0 && !d_tasks)) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "null device buffer");
        }
        CWLB_CUDA(cudaSetDevice(ctx->device));
        *out = cwlb::plan_create(ctx, n_rows, nnz, d_row_offset, d_col_ind, d_value, d_tasks,
                                 n_tasks, group_size);
        return CWLB_OK;
    } catch (const cwlb::Failure& e) {
        cwlb::set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        cwlb::set_last_error(e.what());
        return CWLB_ERR_RUNTIME;
    }
}

int cwlb_plan_info(const cwlb_plan* plan, int64_t* grouped_tasks, int64_t* grouped_nnz,
                   int64_t* union_entries, int32_t* group_size, uint32_t* off_reason) {
    if (!plan) {
        cwlb::set_last_error("null plan");
        return CWLB_ERR_INVALID_ARGUMENT;
    }
    if (grouped_tasks) *grouped_tasks = plan->n_groups > 0 ? plan->grouped_tasks : 0;
    if (grouped_nnz) *grouped_nnz = plan->n_groups > 0 ? plan->grouped_nnz : 0;
    if (union_entries) *union_entries = plan->n_groups > 0 ? plan->union_entries : 0;
    if (group_size) *group_size = plan->R;
    if (off_reason) *off_reason = plan->off_reason;
    return CWLB_OK;
}

int cwlb_plan_aggregate_device(cwlb_plan* plan, const int32_t* d_origin_local, const float* d_H,
                               int64_t h_rows, int64_t K, float* d_out, uint32_t flags) {
    try {
        if (!plan) cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "null plan");
        if (h_rows < 0 || K < 0) cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "negative size");
        if (flags & ~static_cast<uint32_t>(CWLB_ROWS_COVERED | CWLB_DETERMINISTIC)) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "unknown flags");
        }
        if (plan->n_rows > 0 && K > 0 && (!d_out || !d_origin_local || (h_rows > 0 && !d_H))) {
            cwlb::fail(CWLB_ERR_INVALID_ARGUMENT, "null device buffer");
        }
        CWLB_CUDA(cudaSetDevice(plan->ctx->device));
        cwlb::plan_aggregate(plan, d_origin_local, d_H, h_rows, K, d_out, flags);
        return CWLB_OK;
    } catch (const cwlb::Failure& e) {
        cwlb::set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        cwlb::set_last_error(e.what());
        return CWLB_ERR_RUNTIME;
    }
}

int cwlb_plan_destroy(cwlb_plan* plan) {
    cwlb::plan_destroy(plan);
    return CWLB_OK;
}

}  // extern "C"
