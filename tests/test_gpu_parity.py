"""GPU parity: the sm_100a path through the C ABI against the oracle.

Bit-exact: the degree permutation, reordered CSR and task list.
Within REL_TOL (tests/helpers.py): the mean-aggregation output.
"""
import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from conftest import load_npz
from helpers import REL_TOL, assert_mean_close, random_csr, sorted_rowoff_from_degrees

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = cs.Context(0)
    yield c
    c.close()


def test_device_info(ctx):
    info = ctx.device_info()
    assert info["max_work_group_size"] == 1024
    assert info["max_compute_units"] >= 100
    assert info["local_mem_size"] > 0


def _oracle_pipeline(oracle, rowoff, col, val, costs, S):
    origin, srow, scol, sval = oracle.sort_by_degree(rowoff, col, val)
    cap = oracle.capacity_from_s(S, costs)
    tasks = oracle.partition(srow, costs, cap)
    return origin, srow, scol, sval, cap, tasks


def test_cfg1_golden_end_to_end(ctx, oracle):
    g = load_npz("cfg1_er4096.npz")
    rowoff, col = g["rowoff"], g["col"]
    val = np.ones(len(col), np.float32)
    X = graphs.uniform_features_np(4096, 32, seed=0)
    order = ctx.sortCSRByDegree(cs.CSR(rowoff, col, val))
    assert np.array_equal(order.Origin_local, g["origin"])
    assert np.array_equal(order.RowOffset, g["sorted_rowoff"])
    o = oracle.sort_by_degree(rowoff, col, val)
    assert np.array_equal(order.ColInd, o[2]) and np.array_equal(order.Value, o[3])
    costs = cs.SpmmCostParams.from_list(g["costs"])
    cap = cs.capacity_from_s(32, costs)
    assert cap == float(g["capacity"])
    tasks = ctx.costWeightedTaskPartitioning(order, costs, cap)
    assert np.array_equal(tasks, g["tasks"])
    out, t_us = ctx.spmmKernel(order, X, 32, 32, tasks)
    assert t_us > 0
    ref, cond = oracle.spmm_mean_f64(order.RowOffset, order.ColInd, order.Value,
                                     order.Origin_local, X)
    assert_mean_close(out, ref, cond, what="cfg1 vs f64")
    assert_mean_close(out, g["out"].astype(np.float64), cond, tol=2 * REL_TOL, what="cfg1 vs ref")
    assert np.abs(out - g["out"]).max() <= 1e-4  # the reference's own check (utils.h:83)


def test_partition_golden_cases_bit_exact(ctx):
    g = load_npz("partition_cases.npz")
    rp, tp = g["rowoff_ptr"], g["task_ptr"]
    for i in range(len(g["S"])):
        ro = g["rowoff"][rp[i]:rp[i + 1]]
        want = g["tasks"][tp[i]:tp[i + 1]]
        csr = cs.CSR(ro, np.zeros(ro[-1], np.int32), np.zeros(ro[-1], np.float32))
        costs = cs.SpmmCostParams.from_list(g["cost_sets"][g["cset"][i]])
        got = ctx.costWeightedTaskPartitioning(csr, costs, g["capacity"][i])
        assert np.array_equal(got, want), f"partition golden case {i}"


def _partition_case(rng, it):
    n = int(rng.integers(1, 600))
    kind = it % 6
    if kind == 0:
        d = rng.integers(0, 30, n)
    elif kind == 1:
        d = np.minimum((rng.pareto(1.2, n) * 4).astype(int), 3000)
    elif kind == 2:
        d = np.repeat(rng.integers(0, 90, 6), n // 6 + 1)[:n]
    elif kind == 3:
        d = rng.integers(0, 4, n) * rng.integers(0, 50, n)
    elif kind == 4:
        d = np.full(n, int(rng.integers(0, 400)))
    else:
        d = rng.integers(0, 3, n)
    costs = cs.SpmmCostParams(rng.uniform(0.01, 2), rng.uniform(0.01, 2),
                              float(rng.choice([0.0, rng.uniform(-1, 3)])), rng.uniform(0, 6))
    S = int(rng.choice([1, 2, 3, 5, 8, 16, 31, 64, 200, 5000]))
    cap = cs.capacity_from_s(S, costs)
    if it % 7 == 0:
        cap *= rng.uniform(0.1, 3)
    return sorted_rowoff_from_degrees(d), costs, cap


def test_partition_random_vs_oracle(ctx, oracle):
    rng = np.random.default_rng(11)
    for it in range(400):
        ro, costs, cap = _partition_case(rng, it)
        want = oracle.partition(ro, [costs.C_compute_ns, costs.C_load_ns, costs.C_store_ns,
                                     costs.C_atomic_ns], cap)
        csr = cs.CSR(ro, np.zeros(ro[-1], np.int32), np.zeros(ro[-1], np.float32))
        got = ctx.costWeightedTaskPartitioning(csr, costs, cap)
        assert np.array_equal(got, want), f"random partition case {it}"


@pytest.mark.parametrize("costs,cap", [
    ((float("nan"), 1.0, 0.5, 2.0), 40.0),       # non-finite costs: literal path
    ((0.0, 0.0, 0.5, 2.0), 10.0),                # Cc + Cl == 0
    ((-0.5, 0.2, 0.5, 2.0), 10.0),               # Cc + Cl < 0
    ((0.3, 0.4, 0.5, 1.0), float("inf")),        # infinite capacity
    ((0.3, 0.4, 0.5, 1.0), float("nan")),        # NaN capacity
    ((0.3, 0.4, 1e9, 1.0), 50.0),                # every row long, empty rows dropped
    ((0.3, 0.4, 0.0, 1.0), 5.0),                 # zero-weight empty rows
    ((0.3, 0.4, -2.0, 1.0), 5.0),                # negative store cost
])
def test_partition_edge_costs_vs_oracle(ctx, oracle, costs, cap):
    rng = np.random.default_rng(5)
    d = np.concatenate([np.zeros(50, int), rng.integers(1, 40, 300), [500, 2000]])
    ro = sorted_rowoff_from_degrees(d)
    want = oracle.partition(ro, list(costs), cap)
    csr = cs.CSR(ro, np.zeros(ro[-1], np.int32), np.zeros(ro[-1], np.float32))
    got = ctx.costWeightedTaskPartitioning(csr, cs.SpmmCostParams.from_list(costs), cap)
    assert np.array_equal(got, want)


def test_partition_unsorted_rows_vs_oracle(ctx, oracle):
    rng = np.random.default_rng(6)
    for _ in range(30):
        d = rng.integers(0, 120, int(rng.integers(2, 300)))  # not degree-sorted
        ro = np.zeros(len(d) + 1, np.int32)
        ro[1:] = np.cumsum(d)
        costs = [0.2, 0.5, 0.3, 1.0]
        cap = oracle.capacity_from_s(16, costs)
        csr = cs.CSR(ro, np.zeros(ro[-1], np.int32), np.zeros(ro[-1], np.float32))
        got = ctx.costWeightedTaskPartitioning(csr, cs.SpmmCostParams.from_list(costs), cap)
        assert np.array_equal(got, oracle.partition(ro, costs, cap))


@pytest.mark.parametrize("n,maxdeg,hub", [(1, 5, 1), (7, 0, 1), (300, 40, 3), (5000, 20, 70000),
                                          (20000, 300, 50), (70000, 3, 1), (300000, 12, 400),
                                          (1 << 21, 2, 1)])
def test_sort_vs_oracle(ctx, oracle, n, maxdeg, hub):
    rng = np.random.default_rng(n + maxdeg)
    rowoff, col, val = random_csr(rng, n, maxdeg, hubs=1, hub_factor=hub)
    got = ctx.sortCSRByDegree(cs.CSR(rowoff, col, val))
    want = oracle.sort_by_degree(rowoff, col, val)
    assert np.array_equal(got.Origin_local, want[0])
    assert np.array_equal(got.RowOffset, want[1])
    assert np.array_equal(got.ColInd, want[2])
    assert np.array_equal(got.Value, want[3])


@pytest.mark.parametrize("case", ["exact_chunks", "ragged", "hub_only", "row_per_chunk"])
def test_sort_chunk_boundaries(ctx, oracle, case):
    """The row gather cuts the output into 2048-nonzero chunks: rows that end
    or start exactly on a chunk boundary, empty rows between them, a single
    row spanning many chunks and an nnz that is a multiple of the chunk."""
    C = 2048
    rng = np.random.default_rng(len(case))
    if case == "exact_chunks":
        deg = np.array([0, C, 0, 0, C // 2, C // 2, 3 * C, 0, C - 1, 1], np.int64)
    elif case == "ragged":
        deg = np.array([5, 0, C + 7, 0, 2 * C - 3, 11, 0, 1], np.int64)
    elif case == "hub_only":
        deg = np.array([0, 0, 40 * C + 123, 0], np.int64)
    else:
        deg = np.full(64, C, np.int64)
        deg[::3] = 0
    rowoff = np.concatenate([[0], np.cumsum(deg)]).astype(np.int32)
    col = rng.integers(0, len(deg), int(rowoff[-1]), dtype=np.int32)
    val = rng.random(int(rowoff[-1]), dtype=np.float32)
    got = ctx.sortCSRByDegree(cs.CSR(rowoff, col, val))
    want = oracle.sort_by_degree(rowoff, col, val)
    assert np.array_equal(got.Origin_local, want[0])
    assert np.array_equal(got.RowOffset, want[1])
    assert np.array_equal(got.ColInd, want[2])
    assert np.array_equal(got.Value, want[3])


def test_sort_rejects_inconsistent_nnz(ctx):
    with pytest.raises(RuntimeError, match="inconsistent NNZ"):
        ctx.sortCSRByDegree(cs.CSR(np.array([0, 2, 5], np.int32), np.zeros(4, np.int32),
                                   np.zeros(4, np.float32)))


def test_spmm_golden_cases(ctx, oracle):
    g = load_npz("spmm_cases.npz")
    for c in range(int(g["n_cases"])):
        f = {k: g[f"c{c}_{k}"] for k in ("rowoff", "col", "val", "origin", "H", "tasks", "out")}
        K = int(g[f"c{c}_K"])
        order = cs.CSR_Order(f["rowoff"], f["col"], f["val"], f["origin"])
        fn = ctx.spmmKernelLargeKFallback if K > 1024 else ctx.spmmKernel
        out, _ = fn(order, f["H"], K, K, f["tasks"])
        ref, cond = oracle.spmm_mean_f64(f["rowoff"], f["col"], f["val"], f["origin"], f["H"])
        assert_mean_close(out, ref, cond, what=f"golden spmm case {c} K={K}")
        assert_mean_close(out, f["out"].astype(np.float64), cond, tol=2 * REL_TOL,
                          what=f"golden spmm case {c} K={K} vs reference")


KS = [1, 2, 3, 4, 5, 8, 12, 16, 24, 31, 32, 33, 48, 64, 96, 100, 128, 160, 256, 384, 512, 640,
      1000, 1024]


@pytest.mark.parametrize("K", KS)
def test_spmm_random_vs_oracle(ctx, oracle, K):
    rng = np.random.default_rng(K)
    n = 700
    rowoff, col, val = random_csr(rng, n, 60, hubs=2, hub_factor=40)
    H = rng.uniform(-1, 1, (n, K)).astype(np.float32)
    for S in (1, 7, 32, 300):
        costs = [0.1, 0.6, 0.4, 0.9]
        origin, srow, scol, sval, cap, tasks = _oracle_pipeline(oracle, rowoff, col, val, costs, S)
        order = cs.CSR_Order(srow, scol, sval, origin)
        out, _ = ctx.spmmKernel(order, H, K, K, tasks)
        ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, H)
        assert_mean_close(out, ref, cond, what=f"K={K} S={S}")
        o32 = oracle.spmm_mean(srow, scol, sval, origin, H, tasks)
        assert np.abs(out - o32).max() <= 1e-4


@pytest.mark.parametrize("K", [1025, 1100, 1536, 2048, 3001])
def test_spmm_large_k_vs_oracle(ctx, oracle, K):
    rng = np.random.default_rng(K)
    n = 120
    rowoff, col, val = random_csr(rng, n, 50, hubs=1, hub_factor=10)
    H = rng.standard_normal((n, K)).astype(np.float32)
    origin, srow, scol, sval, cap, tasks = _oracle_pipeline(oracle, rowoff, col, val,
                                                            [0.1, 0.6, 0.4, 0.9], 16)
    order = cs.CSR_Order(srow, scol, sval, origin)
    out, _ = ctx.spmmKernelLargeKFallback(order, H, K, K, tasks)
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, H)
    assert_mean_close(out, ref, cond, what=f"large K={K}")


def test_spmm_error_behaviour(ctx):
    order = cs.CSR_Order(np.array([0, 1], np.int32), np.array([0], np.int32),
                         np.ones(1, np.float32), np.zeros(1, np.int32))
    tasks = np.array([[0, 1, 0, 0]], np.int32)
    with pytest.raises(ValueError, match="K <= device max work-group size"):
        ctx.spmmKernel(order, np.ones((1, 1025), np.float32), 0, 1025, tasks)
    with pytest.raises(ValueError, match="requires K > device max work-group size"):
        ctx.spmmKernelLargeKFallback(order, np.ones((1, 64), np.float32), 0, 64, tasks)
    out, t = ctx.spmmKernel(order, np.ones((1, 0), np.float32), 0, 0, tasks)
    assert out.shape == (1, 0) and t == 0.0
    out, t = ctx.spmmKernel(order, np.full((1, 8), 3.0, np.float32), 8, 8,
                            np.zeros((0, 4), np.int32))
    assert not out.any() and t == 0.0
    with pytest.raises(ValueError):
        ctx.spmmKernel(order, np.ones((1, 8), np.float32), 8, 0, tasks)


def test_spmm_bad_indices_raise_without_fault(ctx):
    H = np.ones((4, 16), np.float32)
    good = cs.CSR_Order(np.array([0, 2, 3, 3, 4], np.int32), np.array([0, 1, 2, 3], np.int32),
                        np.ones(4, np.float32), np.array([3, 2, 1, 0], np.int32))
    tasks = np.array([[0, 4, 0, 0]], np.int32)
    bad_col = cs.CSR_Order(good.RowOffset, np.array([0, 9, 2, -1], np.int32), good.Value,
                           good.Origin_local)
    with pytest.raises(ValueError, match="column index"):
        ctx.spmmKernel(bad_col, H, 16, 16, tasks)
    with pytest.raises(ValueError, match="task row"):
        ctx.spmmKernel(good, H, 16, 16, np.array([[0, 9, 0, 0]], np.int32))
    bad_origin = cs.CSR_Order(good.RowOffset, good.ColInd, good.Value,
                              np.array([3, 2, 7, 0], np.int32))
    with pytest.raises(ValueError, match="Origin_local"):
        ctx.spmmKernel(bad_origin, H, 16, 16, tasks)
    out, _ = ctx.spmmKernel(good, H, 16, 16, tasks)  # the context still works
    assert np.allclose(out[[3, 2, 0]], 1.0) and not out[1].any()


@pytest.mark.parametrize("K", [7, 100, 512])
def test_whole_rows_bit_exact(ctx, oracle, K):
    """Widths whose kernels give every row to one lane group (K = 100 and 512:
    one group per warp; K = 7: the scalar kernel) sum a whole row in nonzero
    order with one FMA chain and divide once, exactly as the reference's
    kernel (src/parallelMatrix.cpp:151-236): those rows are bit-identical to
    the oracle's FP32 restatement.  Rows split across tasks differ only in the
    order the fragments are added."""
    rng = np.random.default_rng(100 + K)
    n = 900
    rowoff, col, val = random_csr(rng, n, 70, hubs=3, hub_factor=30)
    H = rng.standard_normal((n, K)).astype(np.float32)
    costs = [0.1, 0.6, 0.4, 0.9]
    # S = 128: all rows but the three hubs are whole inside one task.
    origin, srow, scol, sval, cap, tasks = _oracle_pipeline(oracle, rowoff, col, val, costs, 128)
    order = cs.CSR_Order(srow, scol, sval, origin)
    out, _ = ctx.spmmKernel(order, H, K, K, tasks)
    o32 = oracle.spmm_mean(srow, scol, sval, origin, H, tasks)
    deg = np.diff(srow)
    whole = np.zeros(n, bool)
    for rs, re_, fo, ln in np.asarray(tasks).reshape(-1, 4):
        for r in range(rs, re_):
            b = fo if r == rs else 0
            e = ln if (r == re_ - 1 and ln > 0) else deg[r]
            if b == 0 and e == deg[r]:
                whole[r] = True
    rows = origin[whole]
    assert len(rows) > n // 2
    assert np.array_equal(out[rows], o32[rows])
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, H)
    assert_mean_close(out, ref, cond, what=f"K={K}")


@pytest.mark.parametrize("K", [4, 32, 64, 128, 512])
def test_short_row_mode_vs_oracle(ctx, oracle, K):
    """Many short rows per task (~117 here, >= 16 on average) select the
    kernel's short-row mode (a task's row offsets and origins loaded up front,
    tasks of more than 128 rows falling back per row).  Whole rows of tasks
    with at least 32 rows go to one lane group each: bit-identical to the
    oracle's FP32 restatement; the rest within the tolerance."""
    rng = np.random.default_rng(7 + K)
    n = 6000
    rowoff, col, val = random_csr(rng, n, 4, hubs=2, hub_factor=300)
    H = rng.standard_normal((n, K)).astype(np.float32)
    costs = [0.1, 0.6, 0.4, 0.9]
    origin, srow, scol, sval, cap, tasks = _oracle_pipeline(oracle, rowoff, col, val, costs, 300)
    tk = np.asarray(tasks).reshape(-1, 4)
    assert n >= 16 * len(tk)                      # short-row mode
    assert (tk[:, 1] - tk[:, 0] > 128).any()      # and some tasks beyond the staging size
    order = cs.CSR_Order(srow, scol, sval, origin)
    out, _ = ctx.spmmKernel(order, H, K, K, tasks)
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, H)
    assert_mean_close(out, ref, cond, what=f"K={K}")
    o32 = oracle.spmm_mean(srow, scol, sval, origin, H, tasks)
    deg = np.diff(srow)
    exact = []
    for rs, re_, fo, ln in tk:
        if re_ - rs < 32:
            continue
        for r in range(rs, re_):
            b = fo if r == rs else 0
            e = ln if (r == re_ - 1 and ln > 0) else deg[r]
            if b == 0 and e == deg[r]:
                exact.append(origin[r])
    assert len(exact) > n // 2
    assert np.array_equal(out[exact], o32[exact])


def test_empty_graphs(ctx, oracle):
    """No rows, and rows without nonzeros, through sort, partition and
    aggregation: the same (empty or all-zero) results as the oracle."""
    costs = cs.SpmmCostParams(0.1, 0.6, 0.4, 0.9)
    # No rows at all.
    empty = cs.CSR(np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32))
    order = ctx.sortCSRByDegree(empty)
    assert len(order.Origin_local) == 0
    tasks = ctx.costWeightedTaskPartitioning(order, costs, cs.capacity_from_s(8, costs))
    assert len(tasks) == 0
    # Rows without nonzeros.
    ro = np.zeros(37, np.int32)
    csr = cs.CSR(ro, np.zeros(0, np.int32), np.zeros(0, np.float32))
    order = ctx.sortCSRByDegree(csr)
    o = oracle.sort_by_degree(ro, np.zeros(0, np.int32), np.zeros(0, np.float32))
    assert np.array_equal(order.Origin_local, o[0]) and np.array_equal(order.RowOffset, o[1])
    cap = cs.capacity_from_s(8, costs)
    tasks = ctx.costWeightedTaskPartitioning(order, costs, cap)
    want = oracle.partition(o[1], [0.1, 0.6, 0.4, 0.9], cap)
    assert np.array_equal(tasks, want)
    out, _ = ctx.spmmKernel(order, np.ones((36, 8), np.float32), 8, 8, tasks)
    assert out.shape == (36, 8) and not out.any()


def test_unit_values_are_not_copied_but_give_the_same_result(ctx, oracle):
    """Host-buffer calls whose values are all 1.0 (what the reference's loader
    produces) do not copy the values: a device array of ones stands in.  The
    result is the same as the oracle's; a single other value anywhere (start,
    thread-chunk boundaries, end of a multi-million array) is detected."""
    # A small unit-valued call first; the large ones below grow the array of ones.
    small = cs.CSR_Order(np.array([0, 2, 3], np.int32), np.array([0, 1, 1], np.int32),
                         np.ones(3, np.float32), np.array([1, 0], np.int32))
    out, _ = ctx.spmmKernel(small, np.arange(8, dtype=np.float32).reshape(2, 4), 4, 4,
                            np.array([[0, 2, 0, 0]], np.int32))
    assert np.array_equal(out, np.array([[4, 5, 6, 7], [2, 3, 4, 5]], np.float32))
    rng = np.random.default_rng(77)
    n, K = 40000, 32
    rowoff, col, _ = random_csr(rng, n, 150, hubs=2, hub_factor=20)
    nnz = len(col)
    assert nnz > 2_000_000
    H = rng.standard_normal((n, K)).astype(np.float32)
    costs = [0.1, 0.6, 0.4, 0.9]
    ones = np.ones(nnz, np.float32)
    origin, srow, scol, sval, cap, tasks = _oracle_pipeline(oracle, rowoff, col, ones, costs, 128)
    for pos in [None, 0, nnz // 3, nnz // 2, (2 * nnz) // 3, nnz - 1]:
        v = sval.copy()
        if pos is not None:
            v[pos] = 2.0
        order = cs.CSR_Order(srow, scol, v, origin)
        out, _ = ctx.spmmKernel(order, H, K, K, tasks)
        ref, cond = oracle.spmm_mean_f64(srow, scol, v, origin, H)
        assert_mean_close(out, ref, cond, what=f"pos={pos}")
        o32 = oracle.spmm_mean(srow, scol, v, origin, H, tasks)
        assert np.abs(out - o32).max() <= 1e-4


@pytest.mark.parametrize("unit,K,S", [(True, 16, 256), (False, 16, 256), (True, 1100, 256),
                                      (True, 16, 16), (False, 64, 8)])
def test_chunked_host_call_matches_single_shot(ctx, oracle, unit, K, S):
    """Host-buffer calls of 4M+ nonzeros with tasks in partition order copy
    their nonzeros in chunks and aggregate each chunk as soon as it arrives.
    The same tasks in reverse order cannot be chunked (one copy, one launch):
    both give the oracle's result, and whole rows agree bit for bit.  At
    S = 16 and 8 every chunk runs warp runs of small tasks with the whole
    list's run length."""
    rng = np.random.default_rng(91 if unit else 92)
    n = 50000
    rowoff, col, val = random_csr(rng, n, 200, hubs=3, hub_factor=50)
    if unit:
        val = np.ones_like(val)
    assert len(col) >= (1 << 22)
    H = rng.standard_normal((n, K)).astype(np.float32)
    costs = [0.1, 0.6, 0.4, 0.9]
    origin, srow, scol, sval, cap, tasks = _oracle_pipeline(oracle, rowoff, col, val, costs, S)
    tk = np.asarray(tasks).reshape(-1, 4)
    order = cs.CSR_Order(srow, scol, sval, origin)
    call = ctx.spmmKernel if K <= 1024 else ctx.spmmKernelLargeKFallback
    chunked, t1 = call(order, H, K, K, tk)
    single, t2 = call(order, H, K, K, np.ascontiguousarray(tk[::-1]))
    assert t1 > 0 and t2 > 0
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, H)
    assert_mean_close(chunked, ref, cond, what="chunked")
    assert_mean_close(single, ref, cond, what="single")
    deg = np.diff(srow)
    whole = [origin[r] for rs, re_, fo, ln in tk for r in range(rs, re_)
             if (fo if r == rs else 0) == 0 and (ln if (r == re_ - 1 and ln > 0) else deg[r]) == deg[r]]
    assert np.array_equal(chunked[whole], single[whole])


def _pinned_copy(a):
    torch = pytest.importorskip("torch")
    t = torch.empty(a.shape, dtype=getattr(torch, str(a.dtype)), pin_memory=True)
    out = t.numpy()
    out[...] = a
    return out, t


def test_pageable_and_pinned_host_buffers_agree(ctx, oracle):
    """Large host-buffer calls copy ordinary (pageable) memory through the
    context's ring of four 32 MiB pinned slots, filled and drained by host
    threads, and pinned memory directly.  With 160 MB column arrays (the ring
    wraps) both give the oracle's degree sort bit for bit, and the aggregation
    agrees between them on whole rows bit for bit and elsewhere to rounding."""
    rng = np.random.default_rng(2024)
    n = 400000
    rowoff, col, val = random_csr(rng, n, 200, hubs=2, hub_factor=20)
    assert col.nbytes > 4 * (32 << 20)
    want = oracle.sort_by_degree(rowoff, col, val)
    pinned = [_pinned_copy(a) for a in (rowoff, col, val)]
    for ro_, col_, val_ in ((rowoff, col, val), tuple(p[0] for p in pinned)):
        got = ctx.sortCSRByDegree(cs.CSR(ro_, col_, val_))
        assert np.array_equal(got.Origin_local, want[0])
        assert np.array_equal(got.RowOffset, want[1])
        assert np.array_equal(got.ColInd, want[2])
        assert np.array_equal(got.Value, want[3])
    origin, srow, scol, sval = want
    K = 16
    H = rng.standard_normal((n, K)).astype(np.float32)
    costs = cs.SpmmCostParams.from_list([0.1, 0.6, 0.4, 0.9])
    order = cs.CSR_Order(srow, scol, sval, origin)
    tasks = ctx.costWeightedTaskPartitioning(order, costs, cs.capacity_from_s(512, costs))
    pageable_out, _ = ctx.spmmKernel(order, H, K, K, tasks)  # fresh (untouched) result pages
    held = [_pinned_copy(a) for a in (srow, scol, sval, origin, H, np.zeros((n, K), np.float32))]
    p_order = cs.CSR_Order(*(h[0] for h in held[:4]))
    p_out = held[5][0]
    ctx.spmmKernel(p_order, held[4][0], K, K, tasks, out=p_out)
    deg = np.diff(srow)
    whole = [origin[r] for rs, re_, fo, ln in tasks for r in range(rs, re_)
             if (fo if r == rs else 0) == 0 and (ln if (r == re_ - 1 and ln > 0) else deg[r]) == deg[r]]
    assert len(whole) > n // 2
    assert np.array_equal(pageable_out[whole], p_out[whole])
    np.testing.assert_allclose(pageable_out, p_out, rtol=1e-5, atol=1e-6)
