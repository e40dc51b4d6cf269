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


# ---------------------------------------------------------------------------
# The re-weighted cut (cwlb_shard_bounds_rebalance): every row of old shard g
# weighs its whole-row weight times t[g] / W[g], W[g] the shard's summed
# weight (sequential float64), and the cut rule above runs on that prefix.

def _numpy_rebalance(rowoff, costs, bounds, times):
    deg = np.diff(np.asarray(rowoff, np.int64)).astype(np.float64)
    w = deg * (costs.C_compute_ns + costs.C_load_ns) + costs.C_store_ns
    G = len(bounds) - 1
    scale = np.ones(G)
    for g in range(G):
        seg = w[bounds[g]:bounds[g + 1]]
        W = float(np.cumsum(seg)[-1]) if len(seg) else 0.0  # sequential sum
        if W > 0:
            scale[g] = times[g] / W
    owner = np.repeat(np.arange(G), np.diff(np.asarray(bounds, np.int64)))
    cum = np.cumsum(w * scale[owner])
    n = len(deg)
    total = float(cum[-1]) if n else 0.0
    b = [0]
    for k in range(1, G):
        b.append(min(int(np.searchsorted(cum, total * k / G)) + 1, n))
    b.append(n)
    return np.maximum.accumulate(np.array(b, np.int32))


def _true_cost(rowoff):
    """A stand-in for a kernel whose short rows cost more than the model says."""
    deg = np.diff(np.asarray(rowoff, np.int64)).astype(np.float64)
    return np.where(deg == 0, 6.0, deg + 17.0)


@pytest.mark.parametrize("G", [2, 3, 4, 8])
def test_rebalance_matches_the_rule(G):
    costs = cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722)
    rng = np.random.default_rng(40 + G)
    for ro in list(_cases())[:3]:
        b = cs.shard_bounds(ro, costs, G)
        times = rng.uniform(0.5, 2.0, G)
        got = cs.shard_bounds_rebalance(ro, costs, b, times)
        want = _numpy_rebalance(ro, costs, b, times)
        assert np.array_equal(got, want), (G, got, want)
        assert got[0] == 0 and got[-1] == len(ro) - 1 and (np.diff(got) >= 0).all()


def test_rebalance_keeps_a_cut_whose_times_match_the_model():
    costs = cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722)
    ro = next(_cases())
    w = np.diff(ro.astype(np.int64)) * (costs.C_compute_ns + costs.C_load_ns) + costs.C_store_ns
    for G in (2, 4, 8):
        b = cs.shard_bounds(ro, costs, G)
        times = np.array([np.cumsum(w[b[g]:b[g + 1]])[-1] for g in range(G)]) * 3.0
        assert np.array_equal(cs.shard_bounds_rebalance(ro, costs, b, times), b)


def test_rebalance_converges_on_a_cost_the_model_misprices():
    # R-MAT ids: low ids hold the hubs, high ids the short and empty rows, as
    # in the extreme-skew configuration.
    costs = cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722)
    ro, _, _ = graphs.rmat_np(15, 400_000, 0.70, 0.10, 0.10, seed=9)
    true = _true_cost(ro)
    for G in (2, 4, 8):
        b = cs.shard_bounds(ro, costs, G)

        def imbalance(bb):
            per = np.array([true[bb[g]:bb[g + 1]].sum() for g in range(G)])
            return per.max() / per.mean()

        start = imbalance(b)
        for _ in range(3):
            t = np.array([true[b[g]:b[g + 1]].sum() for g in range(G)])
            b = cs.shard_bounds_rebalance(ro, costs, b, t)
        # Each round cuts the excess over the mean several times; what is left
        # is of the order of the largest row.
        assert start > 1.1, start
        assert imbalance(b) < 1.05, (G, start, imbalance(b))


def test_rebalance_argument_errors():
    costs = cs.SpmmCostParams(0.1, 0.2, 0.3, 0.4)
    ro = np.array([0, 2, 4, 9, 9], np.int32)
    ok = np.array([0, 2, 4], np.int32)
    with pytest.raises(ValueError):
        cs.shard_bounds_rebalance(ro, costs, ok, [1.0])                 # wrong length
    with pytest.raises(ValueError):
        cs.shard_bounds_rebalance(ro, costs, [0, 3, 2], [1.0, 1.0])      # decreasing
    with pytest.raises(ValueError):
        cs.shard_bounds_rebalance(ro, costs, [0, 2, 3], [1.0, 1.0])      # does not end at n
    with pytest.raises(ValueError):
        cs.shard_bounds_rebalance(ro, costs, ok, [1.0, 0.0])             # zero time
    with pytest.raises(ValueError):
        cs.shard_bounds_rebalance(ro, costs, ok, [1.0, float("nan")])
    # A shard without rows has no weight: its time is not used.
    assert list(cs.shard_bounds_rebalance(ro, costs, [0, 0, 4], [0.0, 1.0])) == \
        list(cs.shard_bounds(ro, costs, 2))
    assert list(cs.shard_bounds_rebalance(np.array([0], np.int32), costs, [0, 0], [1.0, 2.0][:1])) \
        == [0, 0]
