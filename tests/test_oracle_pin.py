"""Pins the CPU oracle (oracle/cwlb_oracle.cpp) to the reference.

Two independent pins:
  * the committed golden fixtures, produced by the reference's own
    functions (tests/golden/gen_golden.py), always checked;
  * the reference's sources compiled into oracle/_ref, checked live on fresh
    seeded inputs when that library exists.
Sort, partition and helper results must match bit for bit.  The SpMM output
must match bit for bit as well: the oracle adds split-row fragments in task
order, which is the order the emulated reference uses.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import graphs
from conftest import GOLDEN, load_npz


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_cfg1_generator_reproduces_fixture_inputs():
    g = load_npz("cfg1_er4096.npz")
    rowoff, col, val = graphs.er_np(4096, 8, seed=0)
    X = graphs.uniform_features_np(4096, 32, seed=0)
    assert np.array_equal(rowoff, g["rowoff"]) and np.array_equal(col, g["col"])
    assert sha(rowoff, col, val, X) == str(g["input_sha"])
    assert 30000 < len(col) < 36000  # ~32.8K nnz, average degree 8


def test_cfg1_oracle_matches_reference_fixture(oracle):
    g = load_npz("cfg1_er4096.npz")
    rowoff, col = g["rowoff"], g["col"]
    val = np.ones(len(col), np.float32)
    X = graphs.uniform_features_np(4096, 32, seed=0)
    origin, srow, scol, sval = oracle.sort_by_degree(rowoff, col, val)
    assert np.array_equal(origin, g["origin"])
    assert np.array_equal(srow, g["sorted_rowoff"])
    cap = oracle.capacity_from_s(32, g["costs"])
    assert cap == float(g["capacity"])
    tasks = oracle.partition(srow, g["costs"], cap)
    assert np.array_equal(tasks, g["tasks"])
    out = oracle.spmm_mean(srow, scol, sval, origin, X, tasks)
    assert np.array_equal(out, g["out"])


def test_partition_oracle_matches_reference_fixture(oracle):
    g = load_npz("partition_cases.npz")
    rp, tp = g["rowoff_ptr"], g["task_ptr"]
    for i in range(len(g["S"])):
        ro = g["rowoff"][rp[i]:rp[i + 1]]
        want = g["tasks"][tp[i]:tp[i + 1]]
        got = oracle.partition(ro, g["cost_sets"][g["cset"][i]], g["capacity"][i])
        assert np.array_equal(got, want), f"partition case {i}"


def test_spmm_oracle_matches_reference_fixture(oracle):
    g = load_npz("spmm_cases.npz")
    for c in range(int(g["n_cases"])):
        f = {k: g[f"c{c}_{k}"] for k in ("rowoff", "col", "val", "origin", "H", "tasks", "out")}
        out = oracle.spmm_mean(f["rowoff"], f["col"], f["val"], f["origin"], f["H"], f["tasks"])
        assert np.array_equal(out, f["out"]), f"spmm case {c} (K={int(g[f'c{c}_K'])})"


def test_helpers_match_reference_fixture(oracle):
    with open(os.path.join(GOLDEN, "helpers.json")) as fh:
        h = json.load(fh)
    g = load_npz("partition_cases.npz")
    for s, ci, cap in h["capacity_from_s"]:
        assert oracle.capacity_from_s(s, g["cost_sets"][ci]) == cap
    assert oracle.capacity_from_s(5, [0.0, 0.0, 1.0, 2.5]) == h["capacity_from_s_zero_edge"]
    assert oracle.capacity_from_s(5, [-1.0, 0.5, 1.0, -2.5]) == h["capacity_from_s_neg_edge"]
    for nnz, w in h["recommended_w"]:
        assert oracle.recommended_w(nnz) == w
    for nnz, cu, w, s in h["wave_based_s"]:
        assert oracle.wave_based_s(nnz, cu, w) == s
    f = oracle.features(33, 17)
    assert sha(f) == h["features_33x17_sha256"]


def test_oracle_f64_reference_agrees(oracle):
    g = load_npz("cfg1_er4096.npz")
    X = graphs.uniform_features_np(4096, 32, seed=0)
    rowoff, col = g["rowoff"], g["col"]
    val = np.ones(len(col), np.float32)
    origin, srow, scol, sval = oracle.sort_by_degree(rowoff, col, val)
    ref, cond = oracle.spmm_mean_f64(srow, scol, sval, origin, X)
    err = np.abs(g["out"] - ref) / np.maximum(np.maximum(np.abs(ref), cond), 1e-30)
    assert err.max() < 1e-6


# ---------------------------------------------------------------------------
# live pins against the reference's compiled sources

def _rand_csr(rng, n, maxdeg):
    deg = rng.integers(0, maxdeg + 1, n)
    deg[rng.random(n) < 0.1] = 0
    if n > 3:
        deg[rng.integers(0, n)] = maxdeg * 7
    rowoff = np.zeros(n + 1, np.int32)
    rowoff[1:] = np.cumsum(deg)
    col = rng.integers(0, n, rowoff[-1]).astype(np.int32)
    val = rng.standard_normal(rowoff[-1]).astype(np.float32)
    return rowoff, col, val


@pytest.mark.parametrize("seed", range(4))
def test_oracle_matches_reference_live(oracle, reference, seed):
    rng = np.random.default_rng(1000 + seed)
    for _ in range(40):
        n = int(rng.integers(1, 250))
        rowoff, col, val = _rand_csr(rng, n, int(rng.integers(1, 60)))
        a = oracle.sort_by_degree(rowoff, col, val)
        b = reference.sort_by_degree(rowoff, col, val)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)
        costs = np.array([rng.uniform(0.01, 3), rng.uniform(0.01, 3), rng.uniform(-0.5, 3),
                          rng.uniform(0, 5)])
        S = int(rng.integers(1, 40))
        cap = oracle.capacity_from_s(S, costs)
        assert cap == reference.capacity_from_s(S, costs)
        ta = oracle.partition(a[1], costs, cap)
        assert np.array_equal(ta, reference.partition(a[1], costs, cap))
        K = int(rng.choice([1, 3, 8, 32, 33]))
        H = rng.uniform(-1, 1, (n, K)).astype(np.float32)
        oa = oracle.spmm_mean(a[1], a[2], a[3], a[0], H, ta)
        ob, _ = reference.spmm(a[1], a[2], a[3], a[0], H, ta)
        assert np.array_equal(oa, ob)


def test_oracle_matches_reference_large_k_live(oracle, reference):
    rng = np.random.default_rng(7)
    reference.set_device(max_wg=64, sub_group=32, local_mem=1024, compute_units=4)
    try:
        for K in (65, 128, 129, 192, 300):  # feature rounds T = 2, 2, 3, 3, 5
            rowoff, col, val = _rand_csr(rng, 120, 60)
            a = oracle.sort_by_degree(rowoff, col, val)
            costs = np.array([0.3, 1.2, 0.7, 2.0])
            t = oracle.partition(a[1], costs, oracle.capacity_from_s(16, costs))
            H = rng.uniform(-1, 1, (120, K)).astype(np.float32)
            oa = oracle.spmm_mean(a[1], a[2], a[3], a[0], H, t)
            ob, _ = reference.spmm(a[1], a[2], a[3], a[0], H, t, large_k=True)
            assert np.array_equal(oa, ob)
    finally:
        reference.set_device()


def test_reference_error_behaviour(reference):
    rowoff = np.array([0, 1], np.int32)
    col = np.array([0], np.int32)
    val = np.ones(1, np.float32)
    H = np.ones((1, 2000), np.float32)
    tasks = np.array([[0, 1, 0, 0]], np.int32)
    with pytest.raises(ValueError, match="K <= device max work-group size"):
        reference.spmm(rowoff, col, val, np.zeros(1, np.int32), H, tasks)
    with pytest.raises(ValueError, match="requires K > device max work-group size"):
        reference.spmm(rowoff, col, val, np.zeros(1, np.int32), H[:, :8], tasks, large_k=True)
    out, t = reference.spmm(rowoff, col, val, np.zeros(1, np.int32), H[:, :0], tasks)
    assert out.shape == (1, 0) and t == 0.0
    out, t = reference.spmm(rowoff, col, val, np.zeros(1, np.int32), H[:, :4],
                            np.zeros((0, 4), np.int32))
    assert not out.any() and t == 0.0
