"""GPU tests of the multi-GPU entry points (cwlb_shard_*, cwlb_spmm_mean_multi,
cwlb_gather_rows_multi) through the C ABI.

Each shard is the reference's pipeline applied to a contiguous block of
original rows (main.cpp:197-278 sort, src/utils.cpp:832-1021 partition,
src/parallelMatrix.cpp:151-236 aggregation), so:
  * a shard's permutation-independent results are checked against the oracle
    run on the same block: its task list bit for bit;
  * the assembled output against the oracle's float64 mean of the whole
    graph, within the condition-relative 1e-5 of tests/helpers.py;
  * the shard cuts equal cwlb_shard_bounds, or the cut given explicitly
    (cwlb_shard_create_device_cut, e.g. a cwlb_shard_bounds_rebalance cut).
Most tests run on one B200: two contexts on device 0 are two "GPUs" to the
library (two host threads, two streams), which exercises the sharding, the
threads and the output assembly; the two-GPU test skips on a one-GPU box.
"""
import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from helpers import assert_mean_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

COSTS = cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722)


def _graph(values="normal", K=64):
    ro, col, _ = graphs.rmat_np(14, 300_000, 0.57, 0.19, 0.19, seed=41, symmetrize=True,
                                drop_self_loops=True, dedupe=True)
    rng = np.random.default_rng(42)
    val = (rng.standard_normal(len(col)).astype(np.float32) if values == "normal"
           else np.ones(len(col), np.float32))
    X = graphs.uniform_features_np(len(ro) - 1, K, seed=43)
    return cs.CSR(ro, col, val), X


def _oracle_mean(oracle, csr, X):
    ident = np.arange(csr.rows, dtype=np.int32)
    return oracle.spmm_mean_f64(csr.RowOffset, csr.ColInd, csr.Value, ident, X)


class _DevInt32:
    def __init__(self, ptr, count):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3}


@pytest.mark.parametrize("G,K", [(1, 64), (2, 64), (3, 32), (2, 130)])
def test_multi_entry_point_on_contexts_of_one_gpu(oracle, G, K):
    csr, X = _graph(K=K)
    ctxs = [cs.Context(0) for _ in range(G)]
    try:
        cap = cs.capacity_from_s(48, COSTS)
        out, t_us = cs.spmm_mean_multi(ctxs, csr, X, COSTS, cap)
        assert t_us > 0
        ref, cond = _oracle_mean(oracle, csr, X)
        assert_mean_close(out, ref, cond, what=f"multi G={G} K={K}")
        # Same call again into a caller-supplied buffer: identical rows
        # (each row's fragments come from one shard; atomics order aside,
        # whole rows are deterministic).
        out2 = np.full_like(out, np.nan)
        cs.spmm_mean_multi(ctxs, csr, X, COSTS, cap, out=out2)
        assert_mean_close(out2, ref, cond, what="second call")
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.parametrize("rebalanced", [False, True])
def test_shards_from_device_memory_match_the_oracle_block_by_block(oracle, rebalanced):
    csr, X = _graph()
    G, S = 3, 40
    cap = cs.capacity_from_s(S, COSTS)
    costs_l = [COSTS.C_compute_ns, COSTS.C_load_ns, COSTS.C_store_ns, COSTS.C_atomic_ns]
    bounds = cs.shard_bounds(csr.RowOffset, COSTS, G)
    cut = None
    if rebalanced:  # a cut re-weighted by (made-up) shard times, given explicitly
        cut = cs.shard_bounds_rebalance(csr.RowOffset, COSTS, bounds, [1.0, 2.5, 0.7])
        assert not np.array_equal(cut, bounds)
        bounds = cut
    with cs.Context(0) as ctx:
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        d_ro = torch.from_numpy(csr.RowOffset).cuda()
        d_col = torch.from_numpy(csr.ColInd).cuda()
        d_val = torch.from_numpy(csr.Value).cuda()
        d_X = torch.from_numpy(X).cuda()
        out = torch.full((csr.rows, X.shape[1]), float("nan"), device="cuda")
        for s in range(G):
            sh = cs.Shard.from_device(ctx, csr.rows, csr.nnz, d_ro.data_ptr(), d_col.data_ptr(),
                                      d_val.data_ptr(), COSTS, cap, s, G, cut=cut)
            try:
                assert (sh.row_begin, sh.row_end) == (bounds[s], bounds[s + 1])
                a, b = sh.row_begin, sh.row_end
                e0, e1 = csr.RowOffset[a], csr.RowOffset[b]
                assert sh.nnz == e1 - e0
                blk_ro = csr.RowOffset[a:b + 1] - e0
                srow = oracle.sort_by_degree(blk_ro, csr.ColInd[e0:e1], csr.Value[e0:e1])[1]
                want = oracle.partition(srow, costs_l, cap)
                assert sh.n_tasks == len(want)
                got = torch.as_tensor(_DevInt32(sh.tasks_ptr(), 4 * sh.n_tasks), device="cuda")
                assert np.array_equal(got.view(-1, 4).cpu().numpy(), want), f"shard {s} tasks"
                sh.aggregate_device(d_X.data_ptr(), X.shape[0], X.shape[1], out[a:b].data_ptr())
                torch.cuda.synchronize()
            finally:
                sh.close()
        assert ctx.take_device_errors() == 0
    ref, cond = _oracle_mean(oracle, csr, X)
    assert_mean_close(out.cpu().numpy(), ref, cond, what="assembled shards")


def test_host_shards_with_a_given_cut_assemble_the_whole_output(oracle):
    csr, X = _graph(K=32)
    G = 3
    cap = cs.capacity_from_s(48, COSTS)
    cut = cs.shard_bounds_rebalance(csr.RowOffset, COSTS, cs.shard_bounds(csr.RowOffset, COSTS, G),
                                    [0.6, 1.0, 3.0])
    with cs.Context(0) as ctx:
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        d_X = torch.from_numpy(X).cuda()
        out = torch.full((csr.rows, X.shape[1]), float("nan"), device="cuda")
        for s in range(G):
            sh = cs.Shard.from_host(ctx, csr, COSTS, cap, s, G, cut=cut)
            assert (sh.row_begin, sh.row_end) == (cut[s], cut[s + 1])
            sh.aggregate_device(d_X.data_ptr(), X.shape[0], X.shape[1],
                                out[sh.row_begin:sh.row_end].data_ptr())
            torch.cuda.synchronize()
            sh.close()
        assert ctx.take_device_errors() == 0
    ref, cond = _oracle_mean(oracle, csr, X)
    assert_mean_close(out.cpu().numpy(), ref, cond, what="host shards, given cut")


def test_shard_deterministic_flag_gives_identical_outputs():
    csr, X = _graph(K=32)
    with cs.Context(0) as ctx:
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        sh = cs.Shard.from_host(ctx, csr, COSTS, cs.capacity_from_s(8, COSTS), 1, 2)
        d_X = torch.from_numpy(X).cuda()
        outs = []
        for _ in range(2):
            o = torch.zeros((sh.rows, X.shape[1]), device="cuda")
            sh.aggregate_device(d_X.data_ptr(), X.shape[0], X.shape[1], o.data_ptr(),
                                cs.DETERMINISTIC)
            torch.cuda.synchronize()
            outs.append(o.cpu().numpy())
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
        with pytest.raises(ValueError):
            sh.aggregate_device(d_X.data_ptr(), X.shape[0], X.shape[1], o.data_ptr(),
                                cs.ROWS_COVERED)
        sh.close()


def test_multi_argument_errors():
    csr, X = _graph(K=16)
    c0 = cs.Context(0)
    try:
        with pytest.raises(ValueError, match="only once"):
            cs.spmm_mean_multi([c0, c0], csr, X, COSTS, 10.0)
        bad = cs.CSR(csr.RowOffset.copy(), csr.ColInd, csr.Value)
        bad.RowOffset[-1] += 1
        with pytest.raises(RuntimeError, match="Inconsistent NNZ"):
            cs.spmm_mean_multi([c0], bad, X, COSTS, 10.0)
        with pytest.raises(ValueError, match="shard index"):
            cs.Shard.from_host(c0, csr, COSTS, 10.0, 2, 2)
        d_ro = torch.from_numpy(csr.RowOffset).cuda()
        d_col = torch.from_numpy(csr.ColInd).cuda()
        d_val = torch.from_numpy(csr.Value).cuda()
        for bad_cut in ([0, 5, 3], [1, 5, csr.rows], [0, 5, csr.rows - 1]):
            with pytest.raises(ValueError, match="cut must"):
                cs.Shard.from_device(c0, csr.rows, csr.nnz, d_ro.data_ptr(), d_col.data_ptr(),
                                     d_val.data_ptr(), COSTS, 10.0, 0, 2, cut=bad_cut)
            with pytest.raises(ValueError, match="cut must"):
                cs.Shard.from_host(c0, csr, COSTS, 10.0, 1, 2, cut=bad_cut)
        with pytest.raises(ValueError, match="non-decreasing"):
            cs.Shard.from_host(c0, csr, COSTS, 10.0, 0, 3, cut=[0, 9, 5, csr.rows])
    finally:
        c0.close()


def test_gather_rows_between_contexts_of_one_gpu():
    rows, K = 5000, 48
    X = torch.randn(rows, K, device="cuda")
    bounds = np.array([0, 1234, 1234, 5000], np.int32)  # an empty middle shard
    ctxs = [cs.Context(0) for _ in range(3)]
    try:
        bufs = []
        for g in range(3):
            b = torch.full_like(X, float("nan"))
            b[bounds[g]:bounds[g + 1]] = X[bounds[g]:bounds[g + 1]]
            bufs.append(b)
        torch.cuda.synchronize()
        cs.gather_rows_multi(ctxs, [b.data_ptr() for b in bufs], rows, K, bounds)
        for c in ctxs:
            c.synchronize()
        for b in bufs:
            assert torch.equal(b, X)
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multi_entry_point_on_two_gpus(oracle):
    csr, X = _graph(K=128)
    ctxs = [cs.Context(0), cs.Context(1)]
    try:
        out, t_us = cs.spmm_mean_multi(ctxs, csr, X, COSTS, cs.capacity_from_s(64, COSTS))
        assert t_us > 0
        ref, cond = _oracle_mean(oracle, csr, X)
        assert_mean_close(out, ref, cond, what="two GPUs")
        # Row-sharded X rebuilt on both GPUs by peer copies.
        bounds = cs.shard_bounds(csr.RowOffset, COSTS, 2)
        Xt = torch.from_numpy(X)
        bufs = []
        for g in range(2):
            b = torch.full(X.shape, float("nan"), device=f"cuda:{g}")
            b[bounds[g]:bounds[g + 1]] = Xt[bounds[g]:bounds[g + 1]].to(f"cuda:{g}")
            bufs.append(b)
        for g in range(2):
            torch.cuda.synchronize(g)
        cs.gather_rows_multi(ctxs, [b.data_ptr() for b in bufs], X.shape[0], X.shape[1], bounds)
        for c in ctxs:
            c.synchronize()
        for b in bufs:
            assert torch.equal(b.cpu(), Xt)
    finally:
        for c in ctxs:
            c.close()
