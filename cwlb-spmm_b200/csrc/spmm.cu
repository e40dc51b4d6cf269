// Mean-aggregation SpMM over cost-weighted tasks (sm_100a).
//
// Semantics follow spmmKernel / spmmKernelLargeKFallback
// (src/parallelMatrix.cpp:151-236 and :411-664 of the reference): for every
// task and every reordered row r it covers, the fragment [begin, end) of row r
// (begin = first_row_offset on the task's first row, end = last_row_nnz on its
// last row when > 0, both clamped to [0, deg]) is accumulated as
// acc = fma(value, H[col][k], acc) in nnz order, divided by the FULL degree,
// and stored to out[origin[r]][k] if the fragment is the whole row, or added
// atomically otherwise.
//
// B200 mapping (the reference instead gives each task a work-group of K
// work-items and stages the CSR fragment through local memory):
//   * one warp per task, 8 warps per CTA; the hardware block scheduler
//     balances the cost-equalised tasks across the 148 SMs;
//   * the warp is split into G = 32/L lane groups of L lanes; each lane owns V
//     float4 columns of the row (128-bit coalesced gathers of H rows), so a
//     K-wide row is covered by L*V float4 and K > 4*L*V is tiled over
//     blockIdx.y;
//   * tasks with several rows give each group its own row (rows inside a task
//     have near-equal degree because rows are degree-sorted); a single-row
//     task (a long-row fragment) splits its nonzeros over the groups and
//     reduces them with warp shuffles;
//   * U nonzeros are gathered per step so that U*V independent 16-byte loads
//     are in flight per lane before their FMAs; per column the FMA chain
//     keeps nnz order, so whole rows handled by one group round exactly as
//     the reference does;
//   * 1/deg is applied in registers before the single write-back: streaming
//     stores for whole rows, red.global.add.v4.f32 for fragments.
// No tensor cores: the operation is a gather (each nonzero reads a different
// H row), bound by memory, not by a dense contraction.
//
// Safety: indices are checked before use.  A column outside [0, h_rows), a
// task row outside [0, n_rows), non-monotone offsets or an origin outside
// [0, n_rows) never fault: the entry is skipped and a CWLB_DEVERR_* bit is
// raised in the context's device error word.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "scan.cuh"

namespace cwlb {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kThreads = kWarpsPerCta * 32;

struct SpmmArgs {
    const int32_t* __restrict__ rowoff;
    const int32_t* __restrict__ col;
    const float* __restrict__ val;
    const int32_t* __restrict__ origin;
    const float* __restrict__ H;
    const cwlb_task* __restrict__ tasks;
    float* __restrict__ out;
    uint32_t* err;
    int64_t h_rows;
    int64_t K;  // row stride (in floats) of H and out
    int64_t n_tasks;
    int32_t n_rows;
    int32_t nnz;
    int32_t write_empty;  // rows-covered mode: degree-0 rows get explicit zeros
    // Deterministic mode: fragments of split rows go to frag (row
    // frag_pos[2 t + slot] of K floats; slot 0 = the task's first row, 1 = its
    // last) instead of atomics.  nullptr: atomic mode.
    float* __restrict__ frag;
    const int32_t* __restrict__ frag_pos;
    // Optional launch order: warp slot i (i < n_slots) runs task sched[i], an
    // index into [0, n_tasks); nullptr runs task i for every i < n_tasks.
    const int32_t* __restrict__ sched;
    int64_t n_slots;
    // spmm_run_kernel: consecutive tasks per warp.
    int32_t run;
};

__device__ __forceinline__ void raise_err(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

__device__ __forceinline__ float4 fma4(float a, const float4& x, const float4& acc) {
    return make_float4(fmaf(a, x.x, acc.x), fmaf(a, x.y, acc.y), fmaf(a, x.z, acc.z),
                       fmaf(a, x.w, acc.w));
}

__device__ __forceinline__ float4 div4(const float4& a, float d) {
    return make_float4(__fdiv_rn(a.x, d), __fdiv_rn(a.y, d), __fdiv_rn(a.z, d),
                       __fdiv_rn(a.w, d));
}

// Row bookkeeping shared by all kernels.  Returns false when the row has no
// fragment to process (after writing zeros for an empty row if requested).
struct RowFrag {
    int32_t base;   // rowoff[r]
    int32_t deg;
    int32_t begin;  // fragment within the row
    int32_t end;
    int32_t orig;
};

__device__ __forceinline__ int row_fragment(const SpmmArgs& a, int r, const cwlb_task& t,
                                            RowFrag& f) {
    // 0: process, 1: empty row (deg <= 0), 2: nothing to do / invalid
    const int32_t b0 = __ldg(a.rowoff + r);
    const int32_t b1 = __ldg(a.rowoff + r + 1);
    if (b0 < 0 || b1 < b0 || b1 > a.nnz) {
        raise_err(a.err, CWLB_DEVERR_OFFSETS);
        return 2;
    }
    f.orig = __ldg(a.origin + r);
    if (f.orig < 0 || f.orig >= a.n_rows) {
        raise_err(a.err, CWLB_DEVERR_ORIGIN_RANGE);
        return 2;
    }
    f.base = b0;
    f.deg = b1 - b0;
    if (f.deg <= 0) return 1;
    int32_t begin = (r == t.row_start) ? t.first_row_offset : 0;
    int32_t end = f.deg;
    if (r == t.row_end - 1 && t.last_row_nnz > 0) end = t.last_row_nnz;
    begin = min(max(begin, 0), f.deg);
    end = min(max(end, begin), f.deg);
    f.begin = begin;
    f.end = end;
    return begin < end ? 0 : 2;
}

// row_fragment with the row's offsets and origin already at hand.
__device__ __forceinline__ int row_fragment_at(const SpmmArgs& a, int r, const cwlb_task& t,
                                               int32_t b0, int32_t b1, int32_t orig, RowFrag& f) {
    if (b0 < 0 || b1 < b0 || b1 > a.nnz) {
        raise_err(a.err, CWLB_DEVERR_OFFSETS);
        return 2;
    }
    f.orig = orig;
    if (f.orig < 0 || f.orig >= a.n_rows) {
        raise_err(a.err, CWLB_DEVERR_ORIGIN_RANGE);
        return 2;
    }
    f.base = b0;
    f.deg = b1 - b0;
    if (f.deg <= 0) return 1;
    int32_t begin = (r == t.row_start) ? t.first_row_offset : 0;
    int32_t end = f.deg;
    if (r == t.row_end - 1 && t.last_row_nnz > 0) end = t.last_row_nnz;
    begin = min(max(begin, 0), f.deg);
    end = min(max(end, begin), f.deg);
    f.begin = begin;
    f.end = end;
    return begin < end ? 0 : 2;
}

__device__ __forceinline__ bool load_task(const SpmmArgs& a, int64_t t, cwlb_task& tk) {
    // Scalar loads: a caller's task array need only be 4-byte aligned.
    tk.row_start = __ldg(&a.tasks[t].row_start);
    tk.row_end = __ldg(&a.tasks[t].row_end);
    tk.first_row_offset = __ldg(&a.tasks[t].first_row_offset);
    tk.last_row_nnz = __ldg(&a.tasks[t].last_row_nnz);
    if (tk.row_start < 0 || tk.row_end > a.n_rows || tk.row_start > tk.row_end) {
        raise_err(a.err, CWLB_DEVERR_ROW_RANGE);
        return false;
    }
    return true;
}

// ---------------------------------------------------------------------------
// float4 kernel: L lanes per group, V float4 per lane, U nonzeros per step.
//
// Index handling: a group walks its nonzeros in chunks of L.  Each lane loads
// one (col, value) pair of the chunk with a coalesced load and validates it
// (an out-of-range column becomes (0, 0.0f) and raises CWLB_DEVERR_COL_RANGE);
// the pairs are then broadcast inside the group with __shfl_sync, so every
// nonzero costs two shuffles, one wide address multiply-add, V 16-byte loads
// and 4V FMAs.  Loads of a full chunk are unconditional; in a partial chunk
// the slots past its end hold column 0 (valid) and skip the FMA (and, for
// narrow shapes, the load); padding lanes of a partial K tile read a valid
// column and never write.

template <int L, int V>
struct VecCfg {
    static constexpr int G = 32 / L;
    // Nonzeros gathered per step: 4 for one or two float4 per lane (with one
    // float4, 8 in flight cost configuration 5 4% against 4), 2 for wider.
    static constexpr int U0 = V <= 2 ? 4 : 2;
    static constexpr int U = U0 < L ? U0 : L;
    // Rows of at most 64 floats (short-row graphs): partial chunks skip the
    // X loads of their unused slots.  Wider shapes load unconditionally: the
    // predicates cost them registers and an occupancy step.
    static constexpr bool kSkipUnused = L * V <= 16;
};

// Accumulate the nonzeros of chunks starting at `start`, `start + step`, ...
// (each at most L long, ending at `end`) into acc.  All lanes of the group
// execute this with the same arguments.  Per column, the FMA chain follows
// increasing nonzero index within each chunk and chunk order.
//
// kPrefetch: the next chunk's pair is loaded before this chunk's gathers, so
// its latency overlaps them (6% on configuration 5, 1.5% on 2).  Used by the
// <16,1>, <16,2> and <32,1> shapes; wider or narrower shapes gain registers
// and lose an occupancy step.
template <int L, int V, bool kPrefetch, bool kUnit>
__device__ __forceinline__ void gather_chunks(const SpmmArgs& a, int32_t start, int32_t end,
                                              int32_t step, unsigned gmask, int lg,
                                              const float4* const (&hq)[V], const bool (&ok)[V],
                                              uint32_t K4, float4 (&acc)[V]) {
    constexpr int U = VecCfg<L, V>::U;
    [[maybe_unused]] int32_t nc = 0;
    [[maybe_unused]] float nv = 0.0f;
    if constexpr (kPrefetch) {
        if (start < end && lg < min(L, end - start)) {
            nc = __ldg(a.col + start + lg);
            nv = kUnit ? 1.0f : __ldg(a.val + start + lg);
        }
    }
    for (int32_t pos = start; pos < end; pos += step) {
        const int32_t cnt = min(L, end - pos);
        int32_t c = 0;
        float v = 0.0f;
        if constexpr (kPrefetch) {
            if (lg < cnt) {
                c = nc;
                v = nv;
            }
            const int32_t np = pos + step;
            nc = 0;
            nv = 0.0f;
            if (np < end && lg < min(L, end - np)) {
                nc = __ldg(a.col + np + lg);
                nv = kUnit ? 1.0f : __ldg(a.val + np + lg);
            }
            if (lg < cnt && static_cast<uint32_t>(c) >= static_cast<uint64_t>(a.h_rows)) {
                raise_err(a.err, CWLB_DEVERR_COL_RANGE);
                c = 0;
                v = 0.0f;
            }
        } else {
            if (lg < cnt) {
                c = __ldg(a.col + pos + lg);
                v = kUnit ? 1.0f : __ldg(a.val + pos + lg);
                if (static_cast<uint32_t>(c) >= static_cast<uint64_t>(a.h_rows)) {
                    raise_err(a.err, CWLB_DEVERR_COL_RANGE);
                    c = 0;
                    v = 0.0f;
                }
            }
        }

        if (cnt == L) {
#pragma unroll
            for (int u0 = 0; u0 < L; u0 += U) {
                uint32_t cu[U];
                float vu[U];
#pragma unroll
                for (int t = 0; t < U; ++t) {
                    cu[t] = static_cast<uint32_t>(__shfl_sync(gmask, c, u0 + t, L));
                    // Unit values (all 1.0) need no broadcast: fma(1, x, acc)
                    // rounds exactly as acc + x.  (An out-of-range column is
                    // still flagged; its row 0 is then added, not skipped.)
                    vu[t] = kUnit ? 1.0f : __shfl_sync(gmask, v, u0 + t, L);
                }
                float4 x[U][V];
#pragma unroll
                for (int t = 0; t < U; ++t) {
#pragma unroll
                    for (int i = 0; i < V; ++i)
                        x[t][i] = __ldg(hq[i] + static_cast<size_t>(cu[t]) * K4);
                }
#pragma unroll
                for (int t = 0; t < U; ++t) {
#pragma unroll
                    for (int i = 0; i < V; ++i) acc[i] = fma4(vu[t], x[t][i], acc[i]);
                }
            }
        } else {
            for (int32_t u0 = 0; u0 < cnt; u0 += U) {
                uint32_t cu[U];
                float vu[U];
#pragma unroll
                for (int t = 0; t < U; ++t) {
                    const int src = (u0 + t) & (L - 1);
                    cu[t] = static_cast<uint32_t>(__shfl_sync(gmask, c, src, L));
                    vu[t] = kUnit ? 1.0f : __shfl_sync(gmask, v, src, L);
                }
                float4 x[U][V];
#pragma unroll
                for (int t = 0; t < U; ++t) {
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        if (VecCfg<L, V>::kSkipUnused) {
                            x[t][i] = (u0 + t < cnt)
                                          ? __ldg(hq[i] + static_cast<size_t>(cu[t]) * K4)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                        } else {
                            x[t][i] = __ldg(hq[i] + static_cast<size_t>(cu[t]) * K4);
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < U; ++t) {
                    if (u0 + t < cnt) {
#pragma unroll
                        for (int i = 0; i < V; ++i) acc[i] = fma4(vu[t], x[t][i], acc[i]);
                    }
                }
            }
        }
    }
}

template <int V>
__device__ __forceinline__ void write_row(const SpmmArgs& a, const RowFrag& f,
                                          const int64_t (&q)[V], const bool (&ok)[V],
                                          float4 (&acc)[V], int64_t t, int slot) {
    float4* out4 = reinterpret_cast<float4*>(a.out) + static_cast<int64_t>(f.orig) * (a.K >> 2);
    const float d = static_cast<float>(f.deg);
    const bool full = f.begin == 0 && f.end == f.deg;
    if (!full && a.frag != nullptr) {
        const int32_t pos = __ldg(a.frag_pos + 2 * t + slot);
        if (pos < 0) return;
        float4* dst = reinterpret_cast<float4*>(a.frag) + static_cast<int64_t>(pos) * (a.K >> 2);
#pragma unroll
        for (int i = 0; i < V; ++i)
            if (ok[i]) dst[q[i]] = div4(acc[i], d);
        return;
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
        if (!ok[i]) continue;
        const float4 r = div4(acc[i], d);
        if (full) {
            __stcs(out4 + q[i], r);
        } else {
            atomicAdd(out4 + q[i], r);
        }
    }
}

template <int V>
__device__ __forceinline__ void write_zero_row(const SpmmArgs& a, int32_t orig,
                                               const int64_t (&q)[V], const bool (&ok)[V]) {
    float4* out4 = reinterpret_cast<float4*>(a.out) + static_cast<int64_t>(orig) * (a.K >> 2);
#pragma unroll
    for (int i = 0; i < V; ++i)
        if (ok[i]) __stcs(out4 + q[i], make_float4(0.f, 0.f, 0.f, 0.f));
}


// Task lists of at most this many tasks per SM run one CTA per task
// (spmm_cta_kernel) instead of one warp per task.
#ifndef CWLB_CTA_TASK_SMS
#define CWLB_CTA_TASK_SMS 128
#endif
constexpr int kCtaTasksPerSm = CWLB_CTA_TASK_SMS;

// Short-row mode (windows of row offsets and origins held in registers and
// shared by shuffles) for task lists averaging at least this many rows a task.
#ifndef CWLB_STAGE_ROWS
#define CWLB_STAGE_ROWS 16
#endif
constexpr int64_t kStageRowsPerTask = CWLB_STAGE_ROWS;


// Task lists averaging fewer than kRunMaxTaskNnz nonzeros a task run as warp
// runs of about kRunNnz nonzeros (spmm_run_kernel).
#ifndef CWLB_RUN_NNZ
#define CWLB_RUN_NNZ 2048
#endif
constexpr int64_t kRunNnz = CWLB_RUN_NNZ;
constexpr int64_t kRunMaxTaskNnz = 128;

template <int L, int V, bool kStage, bool kUnit>
__global__ void __launch_bounds__(kThreads) spmm_vec_kernel(SpmmArgs a) {
    constexpr int G = VecCfg<L, V>::G;
    const int lane = threadIdx.x & 31;
    const int64_t slot = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
    if (slot >= a.n_slots) return;
    const int64_t t = a.sched ? static_cast<int64_t>(__ldg(a.sched + slot)) : slot;
    if (t < 0 || t >= a.n_tasks) {  // an order entry outside the task list
        if ((threadIdx.x & 31) == 0) raise_err(a.err, CWLB_DEVERR_ROW_RANGE);
        return;
    }
    cwlb_task tk;
    if (!load_task(a, t, tk)) return;

    const int g = lane / L;
    const int lg = lane % L;
    const unsigned gmask = L == 32 ? 0xffffffffu : (((1u << L) - 1u) << (g * L));
    const uint32_t K4 = static_cast<uint32_t>(a.K >> 2);
    const int64_t q0 = static_cast<int64_t>(blockIdx.y) * (L * V);
    const float4* __restrict__ H4 = reinterpret_cast<const float4*>(a.H);
    int64_t q[V];
    bool ok[V];
    const float4* hq[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        q[i] = q0 + lg + i * L;
        ok[i] = q[i] < static_cast<int64_t>(K4);
        // Padding lanes read a valid column (the row's last) and never write.
        hq[i] = H4 + (ok[i] ? q[i] : static_cast<int64_t>(K4) - 1);
    }
    const int n_task_rows = tk.row_end - tk.row_start;

    if (G == 1 || n_task_rows != 1) {
        // Rows go to teams of T groups.  With at least G rows, T = 1: each
        // group takes its own rows and keeps nonzero order.  With fewer rows
        // than groups, a team splits each row's nonzero chunks and reduces
        // them with shuffles, so no group idles.
        int T = 1;
        if (G > 1) {
            while (T * 2 * n_task_rows <= G) T *= 2;
        }
        const int teams = G / T;
        const int team = g / T;
        const int gt = g - team * T;
        const int team_lanes = T * L;
        const unsigned tmask = team_lanes == 32 ? 0xffffffffu
                                                : (((1u << team_lanes) - 1u) << (team * team_lanes));
        constexpr bool kPf = L >= 16 && L * V <= 32;
        if constexpr (kStage) {
            // Short-row mode: rows in windows of 31.  Lane i loads the offset
            // and origin of the window's row i with one coalesced load each;
            // each row's team takes them by shuffle, so no row waits on its
            // own dependent offset loads.
            for (int wb = tk.row_start; wb < tk.row_end; wb += 31) {
                const int wn = min(31, tk.row_end - wb);
                const int32_t w_ro = lane <= wn ? __ldg(a.rowoff + wb + lane) : 0;
                const int32_t w_org = lane < wn ? __ldg(a.origin + wb + lane) : 0;
                for (int i0 = 0; i0 < wn; i0 += teams) {  // warp-uniform
                    const int i = i0 + team;
                    const int src = min(i, 30);
                    const int32_t b0 = __shfl_sync(0xffffffffu, w_ro, src);
                    const int32_t b1 = __shfl_sync(0xffffffffu, w_ro, src + 1);
                    const int32_t og = __shfl_sync(0xffffffffu, w_org, src);
                    if (i >= wn) continue;
                    const int r = wb + i;
                    RowFrag f;
                    const int st = row_fragment_at(a, r, tk, b0, b1, og, f);
                    if (st == 1) {
                        if (a.write_empty && gt == 0) write_zero_row<V>(a, f.orig, q, ok);
                        continue;
                    }
                    if (st != 0) continue;
                    float4 acc[V];
#pragma unroll
                    for (int k = 0; k < V; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                    gather_chunks<L, V, kPf, kUnit>(a, f.base + f.begin + gt * L, f.base + f.end,
                                                    team_lanes, gmask, lg, hq, ok, K4, acc);
                    for (int sh = L; sh < team_lanes; sh <<= 1) {
#pragma unroll
                        for (int k = 0; k < V; ++k) {
                            acc[k].x += __shfl_xor_sync(tmask, acc[k].x, sh);
                            acc[k].y += __shfl_xor_sync(tmask, acc[k].y, sh);
                            acc[k].z += __shfl_xor_sync(tmask, acc[k].z, sh);
                            acc[k].w += __shfl_xor_sync(tmask, acc[k].w, sh);
                        }
                    }
                    if (gt == 0) write_row<V>(a, f, q, ok, acc, t, r == tk.row_start ? 0 : 1);
                }
            }
        } else {
            for (int r = tk.row_start + team; r < tk.row_end; r += teams) {
                RowFrag f;
                const int st = row_fragment(a, r, tk, f);
                if (st == 1) {
                    if (a.write_empty && gt == 0) write_zero_row<V>(a, f.orig, q, ok);
                    continue;
                }
                if (st != 0) continue;
                float4 acc[V];
#pragma unroll
                for (int i = 0; i < V; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                gather_chunks<L, V, kPf, kUnit>(a, f.base + f.begin + gt * L, f.base + f.end,
                                                team_lanes, gmask, lg, hq, ok, K4, acc);
                for (int sh = L; sh < team_lanes; sh <<= 1) {
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        acc[i].x += __shfl_xor_sync(tmask, acc[i].x, sh);
                        acc[i].y += __shfl_xor_sync(tmask, acc[i].y, sh);
                        acc[i].z += __shfl_xor_sync(tmask, acc[i].z, sh);
                        acc[i].w += __shfl_xor_sync(tmask, acc[i].w, sh);
                    }
                }
                if (gt == 0) write_row<V>(a, f, q, ok, acc, t, r == tk.row_start ? 0 : 1);
            }
        }
    } else {
        // One row: the G groups take interleaved chunks, then reduce by
        // shuffles across groups.
        RowFrag f;
        const int st = row_fragment(a, tk.row_start, tk, f);
        if (st == 1) {
            if (a.write_empty && g == 0) write_zero_row<V>(a, f.orig, q, ok);
            return;
        }
        if (st != 0) return;
        float4 acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        gather_chunks<L, V, L >= 16 && L * V <= 32, kUnit>(a, f.base + f.begin + g * L,
                                                           f.base + f.end, 32, gmask, lg, hq, ok,
                                                           K4, acc);
#pragma unroll
        for (int s = L; s < 32; s <<= 1) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                acc[i].x += __shfl_xor_sync(0xffffffffu, acc[i].x, s);
                acc[i].y += __shfl_xor_sync(0xffffffffu, acc[i].y, s);
                acc[i].z += __shfl_xor_sync(0xffffffffu, acc[i].z, s);
                acc[i].w += __shfl_xor_sync(0xffffffffu, acc[i].w, s);
            }
        }
        if (g == 0) write_row<V>(a, f, q, ok, acc, t, 0);
    }
}

// ---------------------------------------------------------------------------
// Runs of small tasks (a small S): one warp per run of a.run consecutive
// tasks.  Consecutive single-row tasks over adjacent nonzeros of the same row
// (a hub row cut into many S-nonzero fragments) accumulate in the warp's
// registers and reach the output with one atomic add per run onto the zeroed
// row (a single task that covers its row whole is stored, as in
// spmm_vec_kernel): a.run times fewer atomics, and a.run times less rounding
// from adding thousands of fragments to one output row in float (at S = 16 a
// row of degree 10^6 receives 62,500 adds).  Every other
// task runs exactly as in spmm_vec_kernel (same lane groups, teams and
// nonzero order), so every row that a single task covers whole is
// bit-identical between the two kernels.

template <int L, int V, bool kUnit>
__global__ void __launch_bounds__(kThreads) spmm_run_kernel(SpmmArgs a) {
    constexpr int G = VecCfg<L, V>::G;
    constexpr bool kPf = L >= 16 && L * V <= 32;
    const int lane = threadIdx.x & 31;
    const int64_t wi = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
    const int64_t t_begin = wi * a.run;
    if (t_begin >= a.n_tasks) return;
    const int64_t t_end = min(t_begin + static_cast<int64_t>(a.run), a.n_tasks);

    const int g = lane / L;
    const int lg = lane % L;
    const unsigned gmask = L == 32 ? 0xffffffffu : (((1u << L) - 1u) << (g * L));
    const uint32_t K4 = static_cast<uint32_t>(a.K >> 2);
    const int64_t q0 = static_cast<int64_t>(blockIdx.y) * (L * V);
    const float4* __restrict__ H4 = reinterpret_cast<const float4*>(a.H);
    int64_t q[V];
    bool ok[V];
    const float4* hq[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        q[i] = q0 + lg + i * L;
        ok[i] = q[i] < static_cast<int64_t>(K4);
        hq[i] = H4 + (ok[i] ? q[i] : static_cast<int64_t>(K4) - 1);
    }

    // The carried row: sums of consecutive single-row tasks on sorted row
    // c_row, nonzeros [cf.begin, cf.end) of it so far.
    float4 cacc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) cacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    RowFrag cf{};
    int32_t c_row = -1;
    int64_t c_task = 0;
    auto flush = [&]() {  // warp-uniform
        if (c_row < 0) return;
#pragma unroll
        for (int sh = L; sh < 32; sh <<= 1) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                cacc[i].x += __shfl_xor_sync(0xffffffffu, cacc[i].x, sh);
                cacc[i].y += __shfl_xor_sync(0xffffffffu, cacc[i].y, sh);
                cacc[i].z += __shfl_xor_sync(0xffffffffu, cacc[i].z, sh);
                cacc[i].w += __shfl_xor_sync(0xffffffffu, cacc[i].w, sh);
            }
        }
        if (g == 0) write_row<V>(a, cf, q, ok, cacc, c_task, 0);
#pragma unroll
        for (int i = 0; i < V; ++i) cacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        c_row = -1;
    };

    for (int64_t t = t_begin; t < t_end; ++t) {
        cwlb_task tk;
        if (!load_task(a, t, tk)) continue;
        const int n_task_rows = tk.row_end - tk.row_start;
        if (n_task_rows == 1) {
            // One row: the G groups take interleaved chunks (as in
            // spmm_vec_kernel), into the carried sums when the task continues
            // the carried row.
            RowFrag f;
            const int st = row_fragment(a, tk.row_start, tk, f);
            if (st == 0) {
                if (c_row != tk.row_start || f.begin != cf.end) {
                    flush();
                    cf = f;
                    c_row = tk.row_start;
                    c_task = t;
                } else {
                    cf.end = f.end;
                    cf.begin = -1;  // several tasks: added atomically onto the zeroed row
                }
                gather_chunks<L, V, kPf, kUnit>(a, f.base + f.begin + g * L, f.base + f.end, 32,
                                                gmask, lg, hq, ok, K4, cacc);
                continue;
            }
            flush();
            if (st == 1 && a.write_empty && g == 0) write_zero_row<V>(a, f.orig, q, ok);
            continue;
        }
        flush();
        // Several rows: teams of T groups, as in spmm_vec_kernel.
        int T = 1;
        if (G > 1) {
            while (T * 2 * n_task_rows <= G) T *= 2;
        }
        const int teams = G / T;
        const int team = g / T;
        const int gt = g - team * T;
        const int team_lanes = T * L;
        const unsigned tmask = team_lanes == 32 ? 0xffffffffu
                                                : (((1u << team_lanes) - 1u) << (team * team_lanes));
        for (int r = tk.row_start + team; r < tk.row_end; r += teams) {
            RowFrag f;
            const int st = row_fragment(a, r, tk, f);
            if (st == 1) {
                if (a.write_empty && gt == 0) write_zero_row<V>(a, f.orig, q, ok);
                continue;
            }
            if (st != 0) continue;
            // The carry is empty here (flushed above): its registers hold
            // this row's sums.
            gather_chunks<L, V, kPf, kUnit>(a, f.base + f.begin + gt * L, f.base + f.end,
                                            team_lanes, gmask, lg, hq, ok, K4, cacc);
            for (int sh = L; sh < team_lanes; sh <<= 1) {
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    cacc[i].x += __shfl_xor_sync(tmask, cacc[i].x, sh);
                    cacc[i].y += __shfl_xor_sync(tmask, cacc[i].y, sh);
                    cacc[i].z += __shfl_xor_sync(tmask, cacc[i].z, sh);
                    cacc[i].w += __shfl_xor_sync(tmask, cacc[i].w, sh);
                }
            }
            if (gt == 0) write_row<V>(a, f, q, ok, cacc, t, r == tk.row_start ? 0 : 1);
#pragma unroll
            for (int i = 0; i < V; ++i) cacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    flush();
}

// ---------------------------------------------------------------------------
// CTA-per-segment variant: one 8-warp CTA per task, for task lists too short
// to fill the GPU with one warp per task (a large S, or a small graph).  A
// single-row task (a hub fragment) is split over all 8·G lane groups of the
// CTA: each warp reduces its groups with shuffles, then warp 0 adds the eight
// warp sums from shared memory in warp order and writes the row once.  The
// rows of a multi-row task go to the warps in turn (row i to warp i mod 8),
// and inside a warp to lane groups or teams as in spmm_vec_kernel, so every
// row that spmm_vec_kernel sums with one group in nonzero order (bit-identical
// to the reference's order) is summed the same way here.

template <int L, int V, bool kUnit>
__global__ void __launch_bounds__(kThreads) spmm_cta_kernel(SpmmArgs a) {
    constexpr int G = VecCfg<L, V>::G;
    constexpr int W = kWarpsPerCta;
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const int64_t slot = blockIdx.x;  // the grid holds exactly n_slots CTAs
    const int64_t t = a.sched ? static_cast<int64_t>(__ldg(a.sched + slot)) : slot;
    if (t < 0 || t >= a.n_tasks) {  // an order entry outside the task list
        if (threadIdx.x == 0) raise_err(a.err, CWLB_DEVERR_ROW_RANGE);
        return;
    }
    cwlb_task tk;
    if (!load_task(a, t, tk)) return;  // the same task for the whole CTA

    const int g = lane / L;
    const int lg = lane % L;
    const unsigned gmask = L == 32 ? 0xffffffffu : (((1u << L) - 1u) << (g * L));
    const uint32_t K4 = static_cast<uint32_t>(a.K >> 2);
    const int64_t q0 = static_cast<int64_t>(blockIdx.y) * (L * V);
    const float4* __restrict__ H4 = reinterpret_cast<const float4*>(a.H);
    int64_t q[V];
    bool ok[V];
    const float4* hq[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        q[i] = q0 + lg + i * L;
        ok[i] = q[i] < static_cast<int64_t>(K4);
        hq[i] = H4 + (ok[i] ? q[i] : static_cast<int64_t>(K4) - 1);
    }
    const int n_task_rows = tk.row_end - tk.row_start;

    // A whole row with one group per warp (G = 1) stays with one group, so
    // that it sums in nonzero order as spmm_vec_kernel does; other single-row
    // tasks are split over the CTA.
    RowFrag f1;
    const int st1 = n_task_rows == 1 ? row_fragment(a, tk.row_start, tk, f1) : 2;
    if (n_task_rows == 1 && !(G == 1 && st1 == 0 && f1.begin == 0 && f1.end == f1.deg)) {
        __shared__ float4 part[W][L * V];
        const RowFrag& f = f1;
        const int st = st1;  // the same for every thread
        if (st == 1) {
            if (a.write_empty && threadIdx.x < L) write_zero_row<V>(a, f.orig, q, ok);
            return;
        }
        if (st != 0) return;
        float4 acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        gather_chunks<L, V, L >= 16 && L * V <= 32, kUnit>(
            a, f.base + f.begin + (w * G + g) * L, f.base + f.end, W * 32, gmask, lg, hq, ok, K4,
            acc);
#pragma unroll
        for (int sh = L; sh < 32; sh <<= 1) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                acc[i].x += __shfl_xor_sync(0xffffffffu, acc[i].x, sh);
                acc[i].y += __shfl_xor_sync(0xffffffffu, acc[i].y, sh);
                acc[i].z += __shfl_xor_sync(0xffffffffu, acc[i].z, sh);
                acc[i].w += __shfl_xor_sync(0xffffffffu, acc[i].w, sh);
            }
        }
        if (g == 0) {
#pragma unroll
            for (int i = 0; i < V; ++i) part[w][lg * V + i] = acc[i];
        }
        __syncthreads();
        if (w == 0 && g == 0) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                float4 sum = part[0][lg * V + i];
                for (int v = 1; v < W; ++v) {
                    const float4 p = part[v][lg * V + i];
                    sum.x += p.x;
                    sum.y += p.y;
                    sum.z += p.z;
                    sum.w += p.w;
                }
                acc[i] = sum;
            }
            write_row<V>(a, f, q, ok, acc, t, 0);
        }
        return;
    }

    // Multi-row task: row i goes to warp i mod W and, inside the warp, to a
    // team of T groups, T chosen from the task's row count as in
    // spmm_vec_kernel (T = 1 with at least G rows: every row summed by one
    // group in nonzero order).
    int T = 1;
    if (G > 1) {
        while (T * 2 * n_task_rows <= G) T *= 2;
    }
    const int teams = G / T;
    const int team = g / T;
    const int gt = g - team * T;
    const int team_lanes = T * L;
    const unsigned tmask = team_lanes == 32 ? 0xffffffffu
                                            : (((1u << team_lanes) - 1u) << (team * team_lanes));
    for (int r = tk.row_start + w + team * W; r < tk.row_end; r += teams * W) {
        RowFrag f;
        const int st = row_fragment(a, r, tk, f);
        if (st == 1) {
            if (a.write_empty && gt == 0) write_zero_row<V>(a, f.orig, q, ok);
            continue;
        }
        if (st != 0) continue;
        float4 acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        gather_chunks<L, V, false, kUnit>(a, f.base + f.begin + gt * L, f.base + f.end,
                                          team_lanes, gmask, lg, hq, ok, K4, acc);
        for (int sh = L; sh < team_lanes; sh <<= 1) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                acc[i].x += __shfl_xor_sync(tmask, acc[i].x, sh);
                acc[i].y += __shfl_xor_sync(tmask, acc[i].y, sh);
                acc[i].z += __shfl_xor_sync(tmask, acc[i].z, sh);
                acc[i].w += __shfl_xor_sync(tmask, acc[i].w, sh);
            }
        }
        if (gt == 0) write_row<V>(a, f, q, ok, acc, t, r == tk.row_start ? 0 : 1);
    }
}

// ---------------------------------------------------------------------------
// Scalar kernel for K not a multiple of 4 or unaligned H / out: one warp per
// task, lane k owns columns k0 + lane + 32*i, rows in sequence.

template <int V>
__global__ void __launch_bounds__(kThreads) spmm_scalar_kernel(SpmmArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
    if (t >= a.n_tasks) return;
    cwlb_task tk;
    if (!load_task(a, t, tk)) return;
    const int64_t k0 = static_cast<int64_t>(blockIdx.y) * (32 * V);
    int64_t kk[V];
    bool ok[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        kk[i] = k0 + lane + 32 * i;
        ok[i] = kk[i] < a.K;
    }
    for (int r = tk.row_start; r < tk.row_end; ++r) {
        RowFrag f;
        const int st = row_fragment(a, r, tk, f);
        float* orow = a.out + static_cast<int64_t>(f.orig) * a.K;
        if (st == 1) {
            if (a.write_empty) {
#pragma unroll
                for (int i = 0; i < V; ++i)
                    if (ok[i]) __stcs(orow + kk[i], 0.0f);
            }
            continue;
        }
        if (st != 0) continue;
        float acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = 0.0f;
        for (int32_t j = f.base + f.begin; j < f.base + f.end; ++j) {
            int32_t c = __ldg(a.col + j);
            float v = a.val ? __ldg(a.val + j) : 1.0f;
            if (static_cast<uint64_t>(c) >= static_cast<uint64_t>(a.h_rows)) {
                raise_err(a.err, CWLB_DEVERR_COL_RANGE);
                c = 0;
                v = 0.0f;
            }
            const float* hrow = a.H + static_cast<int64_t>(c) * a.K;
#pragma unroll
            for (int i = 0; i < V; ++i)
                acc[i] = fmaf(v, ok[i] ? __ldg(hrow + kk[i]) : 0.0f, acc[i]);
        }
        const float d = static_cast<float>(f.deg);
        const bool full = f.begin == 0 && f.end == f.deg;
        float* frow = nullptr;  // deterministic mode: this fragment's scratch row
        if (!full && a.frag != nullptr) {
            const int32_t pos = __ldg(a.frag_pos + 2 * t + (r == tk.row_start ? 0 : 1));
            if (pos < 0) continue;
            frow = a.frag + static_cast<int64_t>(pos) * a.K;
        }
#pragma unroll
        for (int i = 0; i < V; ++i) {
            if (!ok[i]) continue;
            const float r_ = __fdiv_rn(acc[i], d);
            if (full) __stcs(orow + kk[i], r_);
            else if (frow) frow[kk[i]] = r_;
            else atomicAdd(orow + kk[i], r_);
        }
    }
}

// ---------------------------------------------------------------------------
// Rows-covered mode: zero exactly the output rows that are assembled from
// fragments (each such row has one fragment starting at offset 0), before the
// aggregation kernel adds into them.  One thread checks one task; the warp
// then zeroes the flagged rows together with coalesced stores.

__device__ __forceinline__ int32_t first_fragment_row(const SpmmArgs& a, const cwlb_task& tk,
                                                      int r) {
    // Returns origin[r] if row r's fragment in this task starts at 0 and does
    // not cover the whole row; -1 otherwise.
    const int32_t b0 = __ldg(a.rowoff + r);
    const int32_t b1 = __ldg(a.rowoff + r + 1);
    if (b0 < 0 || b1 < b0 || b1 > a.nnz) return -1;
    const int32_t deg = b1 - b0;
    if (deg <= 0) return -1;
    int32_t begin = (r == tk.row_start) ? tk.first_row_offset : 0;
    int32_t end = deg;
    if (r == tk.row_end - 1 && tk.last_row_nnz > 0) end = tk.last_row_nnz;
    begin = min(max(begin, 0), deg);
    end = min(max(end, begin), deg);
    if (!(begin == 0 && end > 0 && end < deg)) return -1;
    const int32_t o = __ldg(a.origin + r);
    return (o >= 0 && o < a.n_rows) ? o : -1;
}

__global__ void __launch_bounds__(kThreads) zero_split_rows_kernel(SpmmArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    int32_t rows_to_zero[2] = {-1, -1};
    if (t < a.n_tasks) {
        const cwlb_task tk{__ldg(&a.tasks[t].row_start), __ldg(&a.tasks[t].row_end),
                           __ldg(&a.tasks[t].first_row_offset), __ldg(&a.tasks[t].last_row_nnz)};
        if (tk.row_start >= 0 && tk.row_end <= a.n_rows && tk.row_start < tk.row_end) {
            rows_to_zero[0] = first_fragment_row(a, tk, tk.row_start);
            if (tk.row_end - 1 != tk.row_start)
                rows_to_zero[1] = first_fragment_row(a, tk, tk.row_end - 1);
        }
    }
    const bool vec = (a.K % 4 == 0) && (reinterpret_cast<uintptr_t>(a.out) % 16 == 0);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        unsigned pending = __ballot_sync(0xffffffffu, rows_to_zero[i] >= 0);
        while (pending) {
            const int src = __ffs(pending) - 1;
            pending &= pending - 1;
            const int32_t o = __shfl_sync(0xffffffffu, rows_to_zero[i], src);
            if (vec) {
                float4* row = reinterpret_cast<float4*>(a.out) + static_cast<int64_t>(o) * (a.K >> 2);
                for (int64_t k = lane; k < (a.K >> 2); k += 32) row[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                float* row = a.out + static_cast<int64_t>(o) * a.K;
                for (int64_t k = lane; k < a.K; k += 32) row[k] = 0.0f;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Deterministic merge of split rows (CWLB_DETERMINISTIC).
//
// Only a task's first and last rows can be partial.  Plan: count each task's
// partial rows (0-2), scan the counts into positions, and record each
// fragment's row in task order; a row split by the partitioner lies in
// consecutive tasks, so its fragments are consecutive.  The aggregation stores
// every fragment's partial mean at its position.  Then each window of 64
// consecutive fragments is summed per row in order, in place at the first
// fragment of each row's piece, and one warp per row adds its pieces in order
// into the zeroed output row.

constexpr int kMergeWindow = 64;

// Bit 0: the task's first row is partial; bit 1: its (different) last row.
// Mirrors row_fragment: rows with bad offsets or origins are never written.
__device__ __forceinline__ int task_partial_rows(const SpmmArgs& a, const cwlb_task& tk) {
    if (tk.row_start < 0 || tk.row_end > a.n_rows || tk.row_start >= tk.row_end) return 0;
    int m = 0;
    for (int s = 0; s < 2; ++s) {
        const int r = s == 0 ? tk.row_start : tk.row_end - 1;
        if (s == 1 && r == tk.row_start) break;
        const int32_t b0 = __ldg(a.rowoff + r), b1 = __ldg(a.rowoff + r + 1);
        if (b0 < 0 || b1 < b0 || b1 > a.nnz) continue;
        const int32_t o = __ldg(a.origin + r);
        if (o < 0 || o >= a.n_rows) continue;
        const int32_t deg = b1 - b0;
        if (deg <= 0) continue;
        int32_t begin = (r == tk.row_start) ? tk.first_row_offset : 0;
        int32_t end = deg;
        if (r == tk.row_end - 1 && tk.last_row_nnz > 0) end = tk.last_row_nnz;
        begin = min(max(begin, 0), deg);
        end = min(max(end, begin), deg);
        if (begin < end && !(begin == 0 && end == deg)) m |= 1 << s;
    }
    return m;
}

__device__ __forceinline__ cwlb_task load_task_raw(const SpmmArgs& a, int64_t t) {
    return cwlb_task{__ldg(&a.tasks[t].row_start), __ldg(&a.tasks[t].row_end),
                     __ldg(&a.tasks[t].first_row_offset), __ldg(&a.tasks[t].last_row_nnz)};
}

__global__ void __launch_bounds__(kThreads) frag_count_kernel(SpmmArgs a, int32_t* cnt) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (t >= a.n_tasks) return;
    cnt[t] = __popc(task_partial_rows(a, load_task_raw(a, t)));
}

__global__ void __launch_bounds__(kThreads)
    frag_place_kernel(SpmmArgs a, const int32_t* __restrict__ cnt, const int32_t* __restrict__ base,
                      int32_t* __restrict__ frag_pos, int32_t* __restrict__ entry_row,
                      int32_t* __restrict__ n_frag) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (t >= a.n_tasks) return;
    const cwlb_task tk = load_task_raw(a, t);
    const int m = task_partial_rows(a, tk);
    int32_t p = base[t];
    frag_pos[2 * t] = (m & 1) ? p : -1;
    if (m & 1) entry_row[p++] = tk.row_start;
    frag_pos[2 * t + 1] = (m & 2) ? p : -1;
    if (m & 2) entry_row[p++] = tk.row_end - 1;
    if (t == a.n_tasks - 1) *n_frag = base[t] + cnt[t];
}

// Warp w sums fragments [64 w, 64 w + 64) per row piece, in order, and leaves
// each piece's sum at the piece's first fragment.
__global__ void __launch_bounds__(kThreads)
    frag_window_kernel(float* __restrict__ frag, const int32_t* __restrict__ entry_row,
                       const int32_t* __restrict__ n_frag, int64_t K) {
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t nf = *n_frag;
    const int64_t i0 = w * kMergeWindow;
    if (i0 >= nf) return;
    const int64_t i1 = min(i0 + kMergeWindow, nf);
    for (int64_t k = lane; k < K; k += 32) {
        int64_t start = i0;
        int32_t row = entry_row[i0];
        float sum = frag[i0 * K + k];
        // Entries read 8 at a time (loads in flight together), summed in order.
        for (int64_t i = i0 + 1; i < i1; i += 8) {
            float v[8];
            int32_t rr[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                rr[u] = (i + u < i1) ? entry_row[i + u] : -1;
                v[u] = (i + u < i1) ? frag[(i + u) * K + k] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (i + u >= i1) break;
                if (rr[u] != row) {
                    frag[start * K + k] = sum;
                    start = i + u;
                    row = rr[u];
                    sum = v[u];
                } else {
                    sum += v[u];
                }
            }
        }
        frag[start * K + k] = sum;
    }
}

// One warp per row's first fragment: its pieces (the first, then one per
// window boundary inside the row's fragment run) added in order.
__global__ void __launch_bounds__(kThreads)
    frag_final_kernel(const float* __restrict__ frag, const int32_t* __restrict__ entry_row,
                      const int32_t* __restrict__ n_frag, const int32_t* __restrict__ origin,
                      int64_t K, int64_t max_frag, float* __restrict__ out) {
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i >= max_frag) return;
    const int64_t nf = *n_frag;
    if (i >= nf) return;
    const int32_t R = entry_row[i];
    if (i > 0 && entry_row[i - 1] == R) return;
    const int32_t o = __ldg(origin + R);  // checked by the plan
    // The row's pieces: its first fragment, then every window boundary inside
    // its run.  Counted once, then read 8 at a time (loads in flight together)
    // and added strictly in order.
    const int64_t p0 = (i / kMergeWindow + 1) * kMergeWindow;
    int64_t n_more = 0;
    while (p0 + n_more * kMergeWindow < nf && entry_row[p0 + n_more * kMergeWindow] == R) ++n_more;
    for (int64_t k = lane; k < K; k += 32) {
        float sum = frag[i * K + k];
        for (int64_t j = 0; j < n_more; j += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                v[u] = (j + u < n_more) ? frag[(p0 + (j + u) * kMergeWindow) * K + k] : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j + u < n_more) sum += v[u];
        }
        // Added onto the zeroed row: exact for a row with one fragment run.
        atomicAdd(out + static_cast<int64_t>(o) * K + k, sum);
    }
}

template <int L, int V>
void launch_vec(const SpmmArgs& a, bool stage, bool per_cta, cudaStream_t s) {
    const int64_t K4 = a.K >> 2;
    const int64_t tiles = ceil_div(K4, L * V);
    if (a.run > 1) {
        dim3 grid(static_cast<unsigned>(ceil_div(ceil_div(a.n_tasks, a.run), kWarpsPerCta)),
                  static_cast<unsigned>(tiles));
        if (a.val == nullptr) {
            spmm_run_kernel<L, V, true><<<grid, kThreads, 0, s>>>(a);
        } else {
            spmm_run_kernel<L, V, false><<<grid, kThreads, 0, s>>>(a);
        }
        return;
    }
    if (per_cta) {
        dim3 grid(static_cast<unsigned>(a.n_slots), static_cast<unsigned>(tiles));
        if (a.val == nullptr) {
            spmm_cta_kernel<L, V, true><<<grid, kThreads, 0, s>>>(a);
        } else {
            spmm_cta_kernel<L, V, false><<<grid, kThreads, 0, s>>>(a);
        }
        return;
    }
    dim3 grid(static_cast<unsigned>(ceil_div(a.n_slots, kWarpsPerCta)),
              static_cast<unsigned>(tiles));
    // Values NULL (every value 1.0): the instances without value loads and
    // broadcasts (12% on configuration 5, 10% on configuration 4's short-row
    // instance).
    if (stage) {
        if (a.val == nullptr) {
            spmm_vec_kernel<L, V, true, true><<<grid, kThreads, 0, s>>>(a);
        } else {
            spmm_vec_kernel<L, V, true, false><<<grid, kThreads, 0, s>>>(a);
        }
    } else if (a.val == nullptr) {
        spmm_vec_kernel<L, V, false, true><<<grid, kThreads, 0, s>>>(a);
    } else {
        spmm_vec_kernel<L, V, false, false><<<grid, kThreads, 0, s>>>(a);
    }
}

template <int L>
void launch_vec_v(int V, const SpmmArgs& a, bool stage, bool per_cta, cudaStream_t s) {
    switch (V) {
        case 1: launch_vec<L, 1>(a, stage, per_cta, s); break;
        case 2: launch_vec<L, 2>(a, stage, per_cta, s); break;
        case 3: launch_vec<L, 3>(a, stage, per_cta, s); break;
        default: launch_vec<L, 4>(a, stage, per_cta, s); break;
    }
}

// Picks (L, V) for K4 float4 columns.  Two widths use shapes measured
// fastest on B200: K = 32 -> <4,2> and K = 128 -> <16,2> (two float4 per lane
// halve the shuffles per nonzero and double the rows in flight; 10% and 2%
// faster than <8,1> and <32,1> on configurations 4 and 2).  K = 64 keeps
// <16,1>: <8,2> was 5% slower on configuration 5, where more rows in flight
// cost L1 hits on its hub rows.  Other widths: the least padding, then the
// widest group (fewest groups per warp).
void pick_vec_shape(int64_t K4, int& L, int& V) {
    if (K4 == 8 || K4 == 32) {
        L = static_cast<int>(K4 / 2);
        V = 2;
        return;
    }
    int64_t best_waste = -1;
    for (int l = 32; l >= 1; l >>= 1) {
        for (int v = 1; v <= 4; ++v) {
            const int64_t span = static_cast<int64_t>(l) * v;
            // One tile whenever it fits; wider rows use full 128-float4 tiles.
            if (K4 > 128 ? span != 128 : span < K4) continue;
            const int64_t tiles = ceil_div(K4, span);
            const int64_t waste = tiles * span - K4;
            if (best_waste < 0 || waste < best_waste) {
                best_waste = waste;
                L = l;
                V = v;
            }
        }
    }
}

}  // namespace

int32_t task_run_length(int64_t nnz, int64_t n_tasks) {
    if (n_tasks <= 0) return 1;
    const int64_t per_task = std::max<int64_t>(1, nnz / n_tasks);
    if (per_task >= kRunMaxTaskNnz) return 1;
    return static_cast<int32_t>(std::min<int64_t>(32, std::max<int64_t>(2, kRunNnz / per_task)));
}

uint32_t task_variant_flag(const cwlb_ctx* ctx, int64_t n_tasks, uint32_t flags) {
    if (flags & (CWLB_TASK_PER_WARP | CWLB_TASK_PER_CTA | kFlagWarpTasks))
        return flags & (CWLB_TASK_PER_WARP | CWLB_TASK_PER_CTA | kFlagWarpTasks);
    return n_tasks <= static_cast<int64_t>(kCtaTasksPerSm) * ctx->props.multiProcessorCount
               ? CWLB_TASK_PER_CTA
               : kFlagWarpTasks;
}

void launch_spmm_mean(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                      const int32_t* col, const float* val, const int32_t* origin,
                      const float* H, int64_t h_rows, int64_t K, const cwlb_task* tasks,
                      int64_t n_tasks, float* out, uint32_t flags, const int32_t* sched,
                      int64_t n_slots, int32_t run) {
    if (K <= 0 || n_rows <= 0) return;
    cudaStream_t s = ctx->stream;
    const bool covered = (flags & CWLB_ROWS_COVERED) != 0;
    if (!covered && !(flags & kFlagOutCleared)) {
        CWLB_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * static_cast<size_t>(n_rows) * K, s));
    }
    if (n_tasks <= 0) return;
    if (nnz > 0 && h_rows <= 0) fail(CWLB_ERR_INVALID_ARGUMENT, "H has no rows but the CSR has nonzeros");

    SpmmArgs a{};
    a.rowoff = rowoff;
    a.col = col;
    a.val = val;
    a.origin = origin;
    a.H = H;
    a.tasks = tasks;
    a.out = out;
    a.err = ctx->d_error_flags;
    a.h_rows = h_rows;
    a.K = K;
    a.n_tasks = n_tasks;
    a.n_rows = n_rows;
    a.nnz = nnz;
    a.write_empty = covered ? 1 : 0;
    a.sched = sched;
    a.n_slots = sched ? n_slots : n_tasks;

    if (covered && !(flags & kFlagSplitZeroed)) {
        dim3 grid(static_cast<unsigned>(ceil_div(n_tasks, kThreads)));
        zero_split_rows_kernel<<<grid, kThreads, 0, s>>>(a);
        CWLB_LAUNCH_CHECK("zero_split_rows_kernel");
    }

    // Deterministic mode: plan the fragment positions (scratch carved from
    // one context buffer, every piece 256-byte aligned).
    const bool det = (flags & CWLB_DETERMINISTIC) != 0;
    int32_t* n_frag = nullptr;
    int32_t* entry_row = nullptr;
    const int64_t max_frag = 2 * n_tasks;
    if (det) {
        if (max_frag >= (int64_t(1) << 31)) {
            fail(CWLB_ERR_INVALID_ARGUMENT, "deterministic mode supports fewer than 2^30 tasks");
        }
        auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
        const size_t nt = static_cast<size_t>(n_tasks), mf = static_cast<size_t>(max_frag);
        const size_t b_cnt = al(4 * nt), b_scan = al(scan_scratch_bytes<int32_t>(n_tasks));
        const size_t b_pos = al(4 * mf), b_nf = 256;
        const size_t b_frag = al(sizeof(float) * mf * static_cast<size_t>(K));
        char* base = static_cast<char*>(
            ctx->det_scratch.ensure(2 * b_cnt + b_scan + 2 * b_pos + b_nf + b_frag));
        int32_t* cnt = reinterpret_cast<int32_t*>(base);
        int32_t* offs = reinterpret_cast<int32_t*>(base + b_cnt);
        void* scan_tmp = base + 2 * b_cnt;
        int32_t* frag_pos = reinterpret_cast<int32_t*>(base + 2 * b_cnt + b_scan);
        entry_row = reinterpret_cast<int32_t*>(base + 2 * b_cnt + b_scan + b_pos);
        n_frag = reinterpret_cast<int32_t*>(base + 2 * b_cnt + b_scan + 2 * b_pos);
        float* frag = reinterpret_cast<float*>(base + 2 * b_cnt + b_scan + 2 * b_pos + b_nf);
        const unsigned g = static_cast<unsigned>(ceil_div(n_tasks, kThreads));
        frag_count_kernel<<<g, kThreads, 0, s>>>(a, cnt);
        CWLB_LAUNCH_CHECK("frag_count_kernel");
        device_exclusive_scan<int32_t>(cnt, offs, n_tasks, scan_tmp, s);
        frag_place_kernel<<<g, kThreads, 0, s>>>(a, cnt, offs, frag_pos, entry_row, n_frag);
        CWLB_LAUNCH_CHECK("frag_place_kernel");
        a.frag = frag;
        a.frag_pos = frag_pos;
    }

    const bool aligned = (reinterpret_cast<uintptr_t>(H) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (K % 4 == 0);
    if (sched && (!aligned || det)) {
        fail(CWLB_ERR_RUNTIME, "internal: a launch order needs the vector kernel, atomic mode");
    }
    if (a.n_slots <= 0) return;
    if (aligned) {
        int L = 32, V = 1;
        pick_vec_shape(K >> 2, L, V);
        // Short-row mode when tasks hold many rows on average (>= 16, e.g.
        // configuration 4's degree-4 rows, ~54 rows per task): each row's
        // offsets would otherwise be a dependent load on its critical path.
        // Graphs with fewer rows per task keep the plain kernel (its
        // next-chunk prefetch and register budget serve their long rows:
        // configurations 3 and 5 were 2% and 5% slower in short-row mode).
        // One CTA per task when one warp per task would leave the GPU's
        // last waves to a few long tasks (task_variant_flag); callers that
        // launch a list in pieces pass the whole list's choice.
        const bool per_cta = (task_variant_flag(ctx, a.n_tasks, flags) & CWLB_TASK_PER_CTA) != 0;
        const bool stage = !per_cta && static_cast<int64_t>(n_rows) >= kStageRowsPerTask * n_tasks;
        // Small tasks (a small S; not forced to one warp per task): runs of
        // tasks per warp, about kRunNnz nonzeros a run, at most 32 tasks
        // (task_run_length; a caller launching one list in pieces passes the
        // whole list's run length).
        if (!per_cta && !stage && !sched && !det && !(flags & CWLB_TASK_PER_WARP)) {
            const int32_t r = run >= 0 ? run : task_run_length(nnz, n_tasks);
            if (r > 1) a.run = r;
        }
        switch (L) {
            case 1: launch_vec_v<1>(V, a, stage, per_cta, s); break;
            case 2: launch_vec_v<2>(V, a, stage, per_cta, s); break;
            case 4: launch_vec_v<4>(V, a, stage, per_cta, s); break;
            case 8: launch_vec_v<8>(V, a, stage, per_cta, s); break;
            case 16: launch_vec_v<16>(V, a, stage, per_cta, s); break;
            default: launch_vec_v<32>(V, a, stage, per_cta, s); break;
        }
        CWLB_LAUNCH_CHECK("spmm_vec_kernel");
    } else {
        const int V = static_cast<int>(std::min<int64_t>(4, ceil_div(K, 32)));
        dim3 grid(static_cast<unsigned>(ceil_div(n_tasks, kWarpsPerCta)),
                  static_cast<unsigned>(ceil_div(K, 32 * V)));
        switch (V) {
            case 1: spmm_scalar_kernel<1><<<grid, kThreads, 0, s>>>(a); break;
            case 2: spmm_scalar_kernel<2><<<grid, kThreads, 0, s>>>(a); break;
            case 3: spmm_scalar_kernel<3><<<grid, kThreads, 0, s>>>(a); break;
            default: spmm_scalar_kernel<4><<<grid, kThreads, 0, s>>>(a); break;
        }
        CWLB_LAUNCH_CHECK("spmm_scalar_kernel");
    }
    if (det) {
        const unsigned gw = static_cast<unsigned>(
            std::max<int64_t>(1, ceil_div(ceil_div(max_frag, kMergeWindow), kWarpsPerCta)));
        frag_window_kernel<<<gw, kThreads, 0, s>>>(a.frag, entry_row, n_frag, K);
        CWLB_LAUNCH_CHECK("frag_window_kernel");
        const unsigned gf = static_cast<unsigned>(ceil_div(max_frag, kWarpsPerCta));
        frag_final_kernel<<<gf, kThreads, 0, s>>>(a.frag, entry_row, n_frag, origin, K, max_frag,
                                                  out);
        CWLB_LAUNCH_CHECK("frag_final_kernel");
    }
}

// ---------------------------------------------------------------------------
// Float64 reference aggregation (cwlb_spmm_mean_reference_device).
//
// Independent of the sort, the partitioner and the task kernels: one warp per
// row of the caller's (unsorted) CSR, each lane owning columns lane, lane+32,
// ... of a 256-column pass; the row's nonzeros are summed in order in double
// and the mean is rounded once to float.

namespace {

constexpr int kRefCols = 8;  // columns per lane and pass (256 per warp)

__global__ void __launch_bounds__(kThreads)
spmm_mean_reference_kernel(const int32_t* __restrict__ rowoff, const int32_t* __restrict__ col,
                           const float* __restrict__ val, const float* __restrict__ H,
                           int64_t h_rows, int64_t K, int32_t n_rows, int32_t nnz,
                           float* __restrict__ out, uint32_t* __restrict__ err) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= n_rows) return;
    int32_t b = rowoff[row], e = rowoff[row + 1];
    if (b < 0 || e < b || e > nnz) {
        if (lane == 0) raise_err(err, CWLB_DEVERR_OFFSETS);
        b = e = 0;
    }
    const int32_t deg = e - b;
    float* orow = out + row * K;
    for (int64_t k0 = 0; k0 < K; k0 += 32 * kRefCols) {
        double acc[kRefCols];
#pragma unroll
        for (int i = 0; i < kRefCols; ++i) acc[i] = 0.0;
        for (int32_t j = b; j < e; ++j) {
            const int32_t c = col[j];
            if (c < 0 || c >= h_rows) {
                if (lane == 0) raise_err(err, CWLB_DEVERR_COL_RANGE);
                continue;
            }
            const double v = static_cast<double>(val[j]);
            const float* xrow = H + static_cast<int64_t>(c) * K;
#pragma unroll
            for (int i = 0; i < kRefCols; ++i) {
                const int64_t k = k0 + lane + 32 * i;
                if (k < K) acc[i] += v * static_cast<double>(xrow[k]);
            }
        }
#pragma unroll
        for (int i = 0; i < kRefCols; ++i) {
            const int64_t k = k0 + lane + 32 * i;
            if (k < K) orow[k] = deg > 0 ? static_cast<float>(acc[i] / static_cast<double>(deg)) : 0.0f;
        }
    }
}

}  // namespace

namespace {
// Sets *other when some value is not exactly 1.0f (compared as bits, so
// -0.0 and NaN payloads count as other values).
__global__ void values_other_kernel(const float* __restrict__ v, size_t count,
                                    unsigned int* __restrict__ other) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    unsigned int acc = 0;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += stride)
        acc |= __float_as_uint(v[i]) ^ 0x3f800000u;
    if (__any_sync(0xffffffffu, acc != 0) && (threadIdx.x & 31) == 0) atomicOr(other, 1u);
}
}  // namespace


bool values_all_one(cwlb_ctx* ctx, const float* d_val, size_t count, unsigned int* d_flag) {
    if (count == 0) return true;
    CWLB_CUDA(cudaMemsetAsync(d_flag, 0, sizeof(unsigned int), ctx->stream));
    const unsigned blocks = static_cast<unsigned>(
        std::min<int64_t>(ceil_div(static_cast<int64_t>(count), kThreads),
                          static_cast<int64_t>(ctx->props.multiProcessorCount) * 8));
    values_other_kernel<<<blocks, kThreads, 0, ctx->stream>>>(d_val, count, d_flag);
    CWLB_LAUNCH_CHECK("values_other_kernel");
    unsigned int h = 0;
    CWLB_CUDA(cudaMemcpyAsync(&h, d_flag, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream));
    CWLB_CUDA(cudaStreamSynchronize(ctx->stream));
    return h == 0;
}

void launch_spmm_mean_reference(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                                const int32_t* col, const float* val, const float* H,
                                int64_t h_rows, int64_t K, float* out) {
    if (n_rows <= 0 || K <= 0) return;
    const unsigned blocks = static_cast<unsigned>(ceil_div(static_cast<int64_t>(n_rows), kWarpsPerCta));
    spmm_mean_reference_kernel<<<blocks, kThreads, 0, ctx->stream>>>(
        rowoff, col, val, H, h_rows, K, n_rows, nnz, out, ctx->d_error_flags);
    CWLB_LAUNCH_CHECK("spmm_mean_reference_kernel");
}

// ---------------------------------------------------------------------------
// Task-list validation (cwlb_tasks_check).

namespace {

__global__ void check_tasks_kernel(const int32_t* __restrict__ rowoff, int32_t n_rows,
                                   int32_t nnz, const cwlb_task* __restrict__ tasks,
                                   int64_t n_tasks, uint32_t* __restrict__ row_seen,
                                   uint32_t* __restrict__ nnz_count,
                                   unsigned long long* __restrict__ bad) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (t >= n_tasks) return;
    const cwlb_task tk = tasks[t];
    if (tk.row_start < 0 || tk.row_end > n_rows || tk.row_start > tk.row_end) {
        if (lane == 0) atomicAdd(bad, 1ull);
        return;
    }
    for (int r = tk.row_start; r < tk.row_end; ++r) {
        if (lane == 0) row_seen[r] = 1u;
        const int32_t b0 = rowoff[r], b1 = rowoff[r + 1];
        if (b0 < 0 || b1 < b0 || b1 > nnz) continue;
        const int32_t deg = b1 - b0;
        if (deg <= 0) continue;
        int32_t begin = (r == tk.row_start) ? tk.first_row_offset : 0;
        int32_t end = deg;
        if (r == tk.row_end - 1 && tk.last_row_nnz > 0) end = tk.last_row_nnz;
        begin = min(max(begin, 0), deg);
        end = min(max(end, begin), deg);
        for (int32_t j = b0 + begin + lane; j < b0 + end; j += 32) atomicAdd(nnz_count + j, 1u);
    }
}

__global__ void count_coverage_kernel(const uint32_t* __restrict__ row_seen, int32_t n_rows,
                                      const uint32_t* __restrict__ nnz_count, int32_t nnz,
                                      unsigned long long* __restrict__ res) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    unsigned long long unc = 0, bad = 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_rows;
         i += stride)
        unc += row_seen[i] == 0u;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nnz;
         i += stride)
        bad += nnz_count[i] != 1u;
    for (int o = 16; o > 0; o >>= 1) {
        unc += __shfl_xor_sync(0xffffffffu, unc, o);
        bad += __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if ((threadIdx.x & 31) == 0) {
        if (unc) atomicAdd(res + 0, unc);
        if (bad) atomicAdd(res + 1, bad);
    }
}

}  // namespace

void run_tasks_check(cwlb_ctx* ctx, int32_t n_rows, int32_t nnz, const int32_t* rowoff,
                     const cwlb_task* tasks, int64_t n_tasks, int64_t* bad_tasks,
                     int64_t* uncovered_rows, int64_t* nnz_errors) {
    cudaStream_t s = ctx->stream;
    // Each piece starts on a 256-byte boundary (the 64-bit counters need
    // 8-byte alignment for their atomics).
    auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    const size_t rows_b = al(sizeof(uint32_t) * static_cast<size_t>(n_rows > 0 ? n_rows : 0));
    const size_t nnz_b = al(sizeof(uint32_t) * static_cast<size_t>(nnz > 0 ? nnz : 0));
    char* base = static_cast<char*>(ctx->check_scratch.ensure(rows_b + nnz_b + 64));
    uint32_t* row_seen = reinterpret_cast<uint32_t*>(base);
    uint32_t* nnz_count = reinterpret_cast<uint32_t*>(base + rows_b);
    unsigned long long* res = reinterpret_cast<unsigned long long*>(base + rows_b + nnz_b);
    CWLB_CUDA(cudaMemsetAsync(base, 0, rows_b + nnz_b + 64, s));
    if (n_tasks > 0) {
        const int64_t threads = n_tasks * 32;
        check_tasks_kernel<<<static_cast<unsigned>(ceil_div(threads, 256)), 256, 0, s>>>(
            rowoff, n_rows, nnz, tasks, n_tasks, row_seen, nnz_count, res + 2);
        CWLB_LAUNCH_CHECK("check_tasks_kernel");
    }
    count_coverage_kernel<<<ctx->props.multiProcessorCount * 4, 256, 0, s>>>(row_seen, n_rows,
                                                                          nnz_count, nnz, res);
    CWLB_LAUNCH_CHECK("count_coverage_kernel");
    unsigned long long h[3];
    CWLB_CUDA(cudaMemcpyAsync(h, res, sizeof(h), cudaMemcpyDeviceToHost, s));
    CWLB_CUDA(cudaStreamSynchronize(s));
    *uncovered_rows = static_cast<int64_t>(h[0]);
    *nnz_errors = static_cast<int64_t>(h[1]);
    *bad_tasks = static_cast<int64_t>(h[2]);
}

}  // namespace cwlb
