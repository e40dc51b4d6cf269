"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs HERE (where the reference checkout exists): it loads
oracle/_ref/libcwlbref.so -- the reference's unmodified sources compiled by
oracle/Makefile against the host stand-ins in oracle/shim/ -- and records
what the reference's own functions return on seeded inputs:

  cfg1_er4096.npz     config 1 end to end: sortCSRByDegreeDPLCPU
                      (main.cpp:197-278), capacity_from_s (main.cpp:281-292),
                      costWeightedTaskPartitioning (src/utils.cpp:832-1021)
                      and spmmKernel (src/parallelMatrix.cpp:63-254)
  partition_cases.npz many small degree sequences x cost sets x S values,
                      including the edge cases the partitioner branches on
  spmm_cases.npz      small graphs with split rows at several K, including
                      K > 1024 through spmmKernelLargeKFallback
  helpers.json        S-selection helpers, deterministic_features samples,
                      cost-file text

Inputs are regenerated from their seeds by cwlb-spmm_b200/graphs.py; each
fixture stores a SHA-256 of its inputs so a change in a generator shows up
as a test failure instead of a silent mismatch.

Usage:  python tests/golden/gen_golden.py
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "cwlb-spmm_b200"))

import graphs  # noqa: E402
from oracle import Reference  # noqa: E402


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def read_costs(path):
    with open(path) as f:
        return np.array([float(x) for x in f.read().split()[:4]])


COSTS = read_costs(os.path.join(HERE, "spmm_costs.txt"))

# Cost sets for the partition sweep: the committed file, the probe set used
# when the partitioner was analysed (Cc=1, Cl=2, Cs=0.5, Ca=3), a store cost
# of zero (zero-weight empty rows), a negative store cost, and a store cost
# above any capacity (every row long).
COST_SETS = [
    COSTS,
    np.array([1.0, 2.0, 0.5, 3.0]),
    np.array([0.25, 0.75, 0.0, 1.5]),
    np.array([0.3, 0.9, -0.4, 0.8]),
    np.array([0.1, 0.1, 1e6, 0.2]),
    np.array([0.013, 0.7707, 0.3301, 0.61]),
]


def case_degrees(rng, kind, n):
    if kind == "uniform":
        d = rng.integers(0, 40, n)
    elif kind == "powerlaw":
        d = np.minimum((rng.pareto(1.3, n) * 3).astype(np.int64), 1500)
    elif kind == "zeros":
        d = rng.integers(0, 3, n) * rng.integers(0, 2, n)
    elif kind == "hubs":
        d = rng.integers(0, 8, n)
        d[rng.integers(0, n, 3)] = rng.integers(300, 3000, 3)
    elif kind == "equal":
        d = np.full(n, int(rng.integers(1, 200)))
    else:  # runs: long runs of equal degree (periodic packing)
        d = np.repeat(rng.integers(0, 120, 8), n // 8 + 1)[:n]
    return np.sort(d).astype(np.int64)


def rowoff_of(degrees):
    r = np.zeros(len(degrees) + 1, np.int64)
    np.cumsum(degrees, out=r[1:])
    return r.astype(np.int32)


def main():
    ref = Reference()
    ref.set_device()  # sm_89-like table: max work-group 1024, sub-group 32
    out = {}

    # ---- config 1 ------------------------------------------------------------
    rowoff, col, val = graphs.er_np(4096, 8, seed=0)
    X = graphs.uniform_features_np(4096, 32, seed=0)
    origin, srow, scol, sval = ref.sort_by_degree(rowoff, col, val)
    cap = ref.capacity_from_s(32, COSTS)
    tasks = ref.partition(srow, COSTS, cap)
    res, _ = ref.spmm(srow, scol, sval, origin, X, tasks)
    np.savez_compressed(
        os.path.join(HERE, "cfg1_er4096.npz"),
        rowoff=rowoff, col=col, input_sha=sha(rowoff, col, val, X), costs=COSTS,
        S=32, capacity=cap, origin=origin, sorted_rowoff=srow, tasks=tasks, out=res)
    print("cfg1: nnz", len(col), "tasks", len(tasks))

    # ---- partition sweep -------------------------------------------------------
    rng = np.random.default_rng(2024)
    all_rowoff, rowoff_ptr, all_tasks, task_ptr, params = [], [0], [], [0], []
    kinds = ["uniform", "powerlaw", "zeros", "hubs", "equal", "runs"]
    for i in range(240):
        kind = kinds[i % len(kinds)]
        n = int(rng.integers(1, 250))
        ro = rowoff_of(case_degrees(rng, kind, n))
        cset = int(rng.integers(0, len(COST_SETS)))
        S = int(rng.choice([1, 2, 3, 7, 16, 32, 33, 64, 128, 1000]))
        if S < 3 and kind in ("powerlaw", "hubs"):
            S += 5
        cap = ref.capacity_from_s(S, COST_SETS[cset])
        if i % 17 == 5:
            cap = cap * 0.37  # capacities not produced by capacity_from_s
        t = ref.partition(ro, COST_SETS[cset], cap)
        all_rowoff.append(ro)
        rowoff_ptr.append(rowoff_ptr[-1] + len(ro))
        all_tasks.append(t.reshape(-1, 4))
        task_ptr.append(task_ptr[-1] + len(t))
        params.append([cset, S, cap])
    np.savez_compressed(
        os.path.join(HERE, "partition_cases.npz"),
        rowoff=np.concatenate(all_rowoff), rowoff_ptr=np.array(rowoff_ptr, np.int64),
        tasks=np.concatenate(all_tasks).astype(np.int32), task_ptr=np.array(task_ptr, np.int64),
        cost_sets=np.stack(COST_SETS), cset=np.array([p[0] for p in params], np.int32),
        S=np.array([p[1] for p in params], np.int32),
        capacity=np.array([p[2] for p in params], np.float64))
    print("partition cases:", len(params), "tasks", task_ptr[-1])

    # ---- SpMM cases ---------------------------------------------------------
    spmm = {}
    specs = [(1, 64, 40, 8), (3, 64, 40, 4), (4, 96, 30, 16), (8, 64, 60, 16), (32, 128, 50, 8),
             (33, 80, 70, 16), (64, 64, 300, 32), (128, 90, 130, 32), (200, 60, 90, 16),
             (512, 32, 100, 32), (1024, 16, 70, 16), (1100, 16, 70, 16), (2048, 10, 80, 16)]
    for ci, (K, n, maxdeg, S) in enumerate(specs):
        crng = np.random.default_rng(100 + ci)
        deg = crng.integers(0, maxdeg, n)
        deg[crng.integers(0, n)] = maxdeg * 5
        ro, cl, vl = graphs.degree_graph_np(deg, n, seed=200 + ci)
        vl = crng.uniform(-2, 2, len(cl)).astype(np.float32)
        H = crng.uniform(-1, 1, (n, K)).astype(np.float32)
        o, sr, sc, sv = ref.sort_by_degree(ro, cl, vl)
        cap = ref.capacity_from_s(S, COSTS)
        t = ref.partition(sr, COSTS, cap)
        res, _ = ref.spmm(sr, sc, sv, o, H, t, large_k=K > 1024)
        spmm[f"c{ci}_K"] = np.int32(K)
        for nm, arr in dict(rowoff=sr, col=sc, val=sv, origin=o, H=H, tasks=t, out=res).items():
            spmm[f"c{ci}_{nm}"] = arr
    spmm["n_cases"] = np.int32(len(specs))
    np.savez_compressed(os.path.join(HERE, "spmm_cases.npz"), **spmm)
    print("spmm cases:", len(specs))

    # ---- helpers -------------------------------------------------------------
    h = {}
    h["capacity_from_s"] = [[s, ci, ref.capacity_from_s(s, COST_SETS[ci])]
                            for s in (-3, 0, 1, 2, 16, 91, 1000, 2**31 - 1)
                            for ci in range(len(COST_SETS))]
    h["capacity_from_s_zero_edge"] = ref.capacity_from_s(5, [0.0, 0.0, 1.0, 2.5])
    h["capacity_from_s_neg_edge"] = ref.capacity_from_s(5, [-1.0, 0.5, 1.0, -2.5])
    nnzs = [0, 1, 99999, 100000, 499999, 500000, 999999, 10**6, 4999999, 5 * 10**6,
            9999999, 10**7, 49999999, 5 * 10**7, 2**31 - 1, 2**40]
    h["recommended_w"] = [[n, ref.recommended_w(n)] for n in nnzs]
    h["wave_based_s"] = []
    for nnz in (0, 1, 32768, 110_000_000, 2**31 - 1):
        ro = np.array([0, nnz], np.int64).astype(np.int32) if nnz < 2**31 else None
        for cu in (1, 80, 148):
            for w in (1, 16, 2048, 8192):
                h["wave_based_s"].append([nnz, cu, w, ref.wave_based_s(ro, cu, w)])
    h["search_bounds"] = [[v, b, list(ref.search_bounds(v, b))]
                          for v in ([10, 20, 40], [1, 2, 4], [5, 5, 5], [100, 300, 301])
                          for b in (0, 1, 2)]
    h["search_by_count"] = [[lo, hi, c, ref.search_grid(lo, hi, c)]
                            for lo, hi, c in ((1, 10, 6), (5, 5, 3), (10, 40, 4), (3, 8, 100),
                                              (1, 2**31 - 1, 7), (7, 9, 1))]
    h["search_by_step"] = [[lo, hi, s, ref.search_grid(lo, hi, s, by_step=True)]
                           for lo, hi, s in ((1, 10, 3), (5, 5, 2), (10, 40, 7), (1, 100, 100))]
    f = ref.features(33, 17)
    h["features_33x17_sha256"] = sha(f)
    h["features_33x17_first"] = [float(x) for x in f.reshape(-1)[:8]]
    path = "/tmp/cwlb_golden_costs.txt"
    ref.save_costs([0.0213501, 0.6847129, 2.5, 1234.5678919], path)
    with open(path) as fh:
        h["cost_file_text"] = fh.read()
    with open(os.path.join(HERE, "helpers.json"), "w") as fh:
        json.dump(h, fh, indent=1)
    print("helpers written")


if __name__ == "__main__":
    main()
