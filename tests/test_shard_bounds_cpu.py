"""The multi-GPU row-shard rule (cwlb_shard_bounds), on CPU.

Shard s of G takes ORIGINAL rows [b[s], b[s+1]); the cut after shard s-1
follows the first row whose inclusive prefix sum of the whole-row weight
(Cc + Cl) * deg + Cs (the weight the reference's partitioner gives a whole
row, src/utils.cpp:850-852) reaches total * s / G.  The library's host code
is compared, cut for cut, with a numpy statement of that rule (sequential
float64 cumulative sum, multiply and add rounded separately), and the shards'
costs are checked to be balanced to within one row.
"""
import numpy as np
import pytest

import cwlb_spmm as cs
import graphs


def _numpy_rule(rowoff, costs, G):
    deg = np.diff(np.asarray(rowoff, np.int64)).astype(np.float64)
    w = deg * (costs.C_compute_ns + costs.C_load_ns) + costs.C_store_ns
    cum = np.cumsum(w)  # sequential (np.add.accumulate)
    n = len(deg)
    total = float(cum[-1]) if n else 0.0
    b = [0]
    for k in range(1, G):
        b.append(min(int(np.searchsorted(cum, total * k / G)) + 1, n))
    b.append(n)
    return np.maximum.accumulate(np.array(b, np.int32))


def _cases():
    rng = np.random.default_rng(31)
    ro, _, _ = graphs.rmat_np(12, 50_000, 0.57, 0.19, 0.19, seed=4, symmetrize=True,
                              drop_self_loops=True, dedupe=True)
    yield ro
    yield graphs.geometric_np(5000, 4, 200, seed=7)[0]
    d = rng.integers(0, 40, 3000)
    d[rng.integers(0, 3000, 5)] = 50_000  # hubs
    ro = np.zeros(len(d) + 1, np.int64)
    ro[1:] = np.cumsum(d)
    yield ro.astype(np.int32)
    yield np.zeros(8, np.int32)                   # empty rows only
    yield np.array([0, 1000], np.int32)           # one row


@pytest.mark.parametrize("G", [1, 2, 3, 4, 8])
def test_shard_bounds_match_the_rule(G):
    costs_sets = [cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722),
                  cs.SpmmCostParams(0.3, 0.1, 0.0, 1.0),
                  cs.SpmmCostParams(0.02, 0.7, 2.5, 0.5)]
    for ro in _cases():
        for costs in costs_sets:
            got = cs.shard_bounds(ro, costs, G)
            want = _numpy_rule(ro, costs, G)
            assert np.array_equal(got, want), (G, costs, got, want)
            assert got[0] == 0 and got[-1] == len(ro) - 1 and (np.diff(got) >= 0).all()


def test_shards_are_balanced_to_within_one_row():
    ro, _, _ = graphs.rmat_np(14, 300_000, 0.57, 0.19, 0.19, seed=8, symmetrize=True,
                              drop_self_loops=True, dedupe=True)
    costs = cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722)
    w = np.diff(ro.astype(np.int64)) * (costs.C_compute_ns + costs.C_load_ns) + costs.C_store_ns
    for G in (2, 4, 8):
        b = cs.shard_bounds(ro, costs, G)
        per = np.array([w[b[s]:b[s + 1]].sum() for s in range(G)])
        assert abs(per - w.sum() / G).max() <= w.max() + 1e-9


def test_shard_bounds_argument_errors():
    costs = cs.SpmmCostParams(0.1, 0.2, 0.3, 0.4)
    with pytest.raises(ValueError):
        cs.shard_bounds(np.array([0, 2, 4], np.int32), costs, 0)
    assert list(cs.shard_bounds(np.array([0], np.int32), costs, 3)) == [0, 0, 0, 0]
