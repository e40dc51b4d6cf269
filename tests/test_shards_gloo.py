"""The N > 1 host logic on CPU: two gloo ranks shard the rows, each runs the
per-shard pipeline (degree sort, partition, aggregation -- the oracle here,
the GPU library on the box), and the gathered slices equal the single-rank
result.  No GPU is used."""
import os
import socket

import numpy as np
import pytest

import graphs
import shards

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

COSTS = [0.02135, 0.684712, 0.298413, 0.517096]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _graph():
    rowoff, col, val = graphs.rmat_np(12, 60_000, 0.57, 0.19, 0.19, seed=5, symmetrize=True,
                                      drop_self_loops=True, dedupe=True)
    X = graphs.uniform_features_np(len(rowoff) - 1, 16, seed=6)
    return rowoff, col, val, X


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "cwlb-spmm_b200")]
        from oracle import Oracle
        oracle = Oracle()
        rowoff, col, val, X = _graph()
        a, b = shards.shard_bounds(rowoff, COSTS[0] + COSTS[1], COSTS[2], world, rank)
        ro, c, v = shards.shard_csr(rowoff, col, val, a, b)
        origin, srow, scol, sval = oracle.sort_by_degree(ro, c, v)
        cap = oracle.capacity_from_s(16, COSTS)
        tasks = oracle.partition(srow, COSTS, cap)
        out = oracle.spmm_mean(srow, scol, sval, origin, X, tasks)
        parts = [None] * world
        dist.all_gather_object(parts, (a, b, out))
        if rank == 0:
            np.save(out_path, np.concatenate([p[2] for p in parts], axis=0))
            bounds = np.array([[p[0], p[1]] for p in parts])
            np.save(out_path + ".bounds.npy", bounds)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_row_shards_reassemble_to_single_rank_result(tmp_path, oracle, world):
    out_path = str(tmp_path / "out.npy")
    mp.spawn(_worker, args=(world, _free_port(), out_path), nprocs=world, join=True)
    gathered = np.load(out_path)
    bounds = np.load(out_path + ".bounds.npy")
    rowoff, col, val, X = _graph()
    n = len(rowoff) - 1
    # contiguous cover of all rows
    assert bounds[0, 0] == 0 and bounds[-1, 1] == n
    assert all(bounds[i, 1] == bounds[i + 1, 0] for i in range(world - 1))
    # cost balance: every shard within one heaviest row of the ideal share
    w = np.diff(rowoff) * (COSTS[0] + COSTS[1]) + COSTS[2]
    share = [w[a:b].sum() for a, b in bounds]
    assert max(share) - min(share) <= 2 * w.max() + 1e-9
    # same result as one rank (whole rows bit-identical, split rows within tolerance)
    origin, srow, scol, sval = oracle.sort_by_degree(rowoff, col, val)
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, X)
    from helpers import assert_mean_close
    assert gathered.shape == ref.shape
    assert_mean_close(gathered, ref, cond, what="sharded vs single")


def _gather_worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rowoff, col, val, X = _graph()
        bounds = [shards.shard_bounds(rowoff, COSTS[0] + COSTS[1], COSTS[2], world, r)
                  for r in range(world)]
        # Each rank starts with only its own block (the rest poisoned).
        x = torch.full(X.shape, float("nan"))
        a, b = bounds[rank]
        x[a:b] = torch.from_numpy(X[a:b])
        shards.gather_rows(x, bounds)
        np.save(out_path + f".{rank}.npy", x.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_rows_rebuilds_the_sharded_input_on_every_rank(tmp_path, world):
    out_path = str(tmp_path / "x")
    mp.spawn(_gather_worker, args=(world, _free_port(), out_path), nprocs=world, join=True)
    _, _, _, X = _graph()
    for r in range(world):
        got = np.load(out_path + f".{r}.npy")
        assert np.array_equal(got, X), f"rank {r}"


def _rebalance_worker(rank, world, port, out_path):
    """The bench's re-cut protocol (bench.py rebalance_shards) with gloo: every
    rank 'times' its own shard (here a stand-in cost that prices short rows
    far above the model), the times are all-gathered, every rank computes the
    re-weighted cut, and the shards of that cut are aggregated and gathered."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "cwlb-spmm_b200")]
        import cwlb_spmm as cs
        from oracle import Oracle
        oracle = Oracle()
        rowoff, col, val, X = _graph()
        costs = cs.SpmmCostParams(*COSTS)
        deg = np.diff(rowoff.astype(np.int64))
        true_cost = np.where(deg == 0, 6.0, deg + 17.0)
        cut = cs.shard_bounds(rowoff, costs, world)
        cuts = [cut.tolist()]
        for _ in range(3):
            t = torch.tensor([float(true_cost[cut[rank]:cut[rank + 1]].sum())], dtype=torch.float64)
            times = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(times, t)
            cut = cs.shard_bounds_rebalance(rowoff, costs, cut, [float(v) for v in times])
            cuts.append(cut.tolist())
        a, b = int(cut[rank]), int(cut[rank + 1])
        ro, c, v = shards.shard_csr(rowoff, col, val, a, b)
        origin, srow, scol, sval = oracle.sort_by_degree(ro, c, v)
        tasks = oracle.partition(srow, COSTS, oracle.capacity_from_s(16, COSTS))
        out = oracle.spmm_mean(srow, scol, sval, origin, X, tasks)
        parts = [None] * world
        dist.all_gather_object(parts, (cuts, out))
        if rank == 0:
            np.save(out_path, np.concatenate([p[1] for p in parts], axis=0))
            np.save(out_path + ".cuts.npy", np.array([p[0] for p in parts]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_rebalanced_cut_is_the_same_on_every_rank(tmp_path, oracle, world):
    out_path = str(tmp_path / "rb.npy")
    mp.spawn(_rebalance_worker, args=(world, _free_port(), out_path), nprocs=world, join=True)
    cuts = np.load(out_path + ".cuts.npy")  # (ranks, rounds + 1, world + 1)
    assert all(np.array_equal(cuts[0], cuts[r]) for r in range(world))
    rowoff, col, val, X = _graph()
    deg = np.diff(rowoff.astype(np.int64))
    true_cost = np.where(deg == 0, 6.0, deg + 17.0)

    def imbalance(c):
        per = np.array([true_cost[c[g]:c[g + 1]].sum() for g in range(world)])
        return per.max() / per.mean()

    assert imbalance(cuts[0][-1]) < imbalance(cuts[0][0])
    origin, srow, scol, sval = oracle.sort_by_degree(rowoff, col, val)
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, X)
    from helpers import assert_mean_close
    assert_mean_close(np.load(out_path), ref, cond, what="re-cut shards vs single")
