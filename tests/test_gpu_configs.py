"""GPU parity on the benchmark configurations themselves (scaled down).

bench.py measures configurations 2-5 of graphs.CONFIGS; this file runs the
same device pipeline the bench times (device degree sort -> device
partitioner -> task check -> cwlb_spmm_mean_device with the bench's flags)
on seeded copies of those configurations, shrunk so that the CPU oracle
finishes in seconds, and checks it against the oracle:

  * permutation and reordered CSR: bit-exact (main.cpp:197-278);
  * task list at each S of the reference's --candidates procedure:
    bit-exact (src/utils.cpp:832-1021);
  * output: within the condition-relative 1e-5 of tests/helpers.py against
    the oracle's float64 mean (src/parallelMatrix.cpp:151-236).

S is chosen from the FULL configuration's nonzero count, so a task holds as
many rows and nonzeros as in the benchmark and the aggregation runs the same
kernel instance (lane shape from K, short-row staging from rows per task).
"""
import os

import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from helpers import assert_mean_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COSTS_FILE = os.path.join(ROOT, "cwlb-spmm_b200", "resources", "spmm_costs.txt")

# (configuration, scale-down factor, whether some candidate S must run the
# short-row staging instance, >= 16 rows per task, as configuration 4 does)
CASES = [(2, 4, False), (3, 16, False), (4, 16, True), (5, 4, False)]


@pytest.fixture(scope="module")
def ctx():
    c = cs.Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


class _DevInt32:
    def __init__(self, ptr, count):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3}


def _full_size_candidates(nnz_full, compute_units):
    ws = cs.recommended_candidate_w(nnz_full)
    return sorted({cs.wave_based_s(nnz_full, compute_units, w) for w in ws})


@pytest.mark.parametrize("cfg,scale,staged", CASES)
def test_benchmark_config_scaled_parity(ctx, oracle, cfg, scale, staged):
    rowoff, col, val, X = graphs.build_config_torch(cfg, "cuda", scale_down=scale)
    n, nnz, K = rowoff.numel() - 1, col.numel(), X.shape[1]
    dev = X.device

    # Device degree sort (cwlb_sort_by_degree_device), as bench.device_prepare.
    org = torch.empty(n, dtype=torch.int32, device=dev)
    sro = torch.empty(n + 1, dtype=torch.int32, device=dev)
    scol = torch.empty(nnz, dtype=torch.int32, device=dev)
    sval = torch.empty(nnz, dtype=torch.float32, device=dev)
    ctx.sort_by_degree_device(n, nnz, rowoff.data_ptr(), col.data_ptr(), val.data_ptr(),
                              org.data_ptr(), sro.data_ptr(), scol.data_ptr(), sval.data_ptr())
    torch.cuda.synchronize()
    ro_h, col_h, val_h = rowoff.cpu().numpy(), col.cpu().numpy(), val.cpu().numpy()
    o_org, o_sro, o_scol, o_sval = oracle.sort_by_degree(ro_h, col_h, val_h)
    assert np.array_equal(org.cpu().numpy(), o_org)
    assert np.array_equal(sro.cpu().numpy(), o_sro)
    assert np.array_equal(scol.cpu().numpy(), o_scol)
    assert np.array_equal(sval.cpu().numpy(), o_sval)

    X_h = X.cpu().numpy()
    ref, cond = oracle.spmm_mean_f64(o_sro, o_scol, o_sval, o_org, X_h)

    costs = cs.read_costs_one_per_line(COSTS_FILE)
    cost_list = [costs.C_compute_ns, costs.C_load_ns, costs.C_store_ns, costs.C_atomic_ns]
    cus = ctx.device_info()["max_compute_units"]
    out = torch.empty((n, K), dtype=torch.float32, device=dev)
    staged_seen = False
    for S in _full_size_candidates(nnz * scale, cus):
        cap = cs.capacity_from_s(S, costs)
        ptr, n_tasks = ctx.partition_device(n, sro.data_ptr(), costs, cap)
        tasks = torch.as_tensor(_DevInt32(ptr, n_tasks * 4), device=dev).clone().view(n_tasks, 4)
        torch.cuda.synchronize()
        want = oracle.partition(o_sro, cost_list, cap)
        assert np.array_equal(tasks.cpu().numpy(), want), f"config {cfg} S={S}: task list"
        # The bench's flags: rows-covered mode once the task list checks out.
        chk = ctx.tasks_check(n, nnz, sro.data_ptr(), tasks.data_ptr(), n_tasks)
        assert chk == dict(bad_tasks=0, uncovered_rows=0, nnz_coverage_errors=0)
        staged_seen |= n >= 16 * n_tasks
        out.fill_(float("nan"))  # every element must be written by the kernels
        ctx.spmm_mean_device(n, nnz, sro.data_ptr(), scol.data_ptr(), sval.data_ptr(),
                             org.data_ptr(), X.data_ptr(), X.shape[0], K, tasks.data_ptr(),
                             n_tasks, out.data_ptr(), cs.ROWS_COVERED)
        torch.cuda.synchronize()
        assert ctx.take_device_errors() == 0
        assert_mean_close(out.cpu().numpy(), ref, cond,
                          what=f"config {cfg} / {scale} S={S} ({n_tasks} tasks)")
    if staged:
        assert staged_seen, "no candidate S reached the short-row staging instance"


@pytest.mark.parametrize("cfg", [2, 3, 4, 5])
def test_benchmark_config_full_size(ctx, cfg):
    """The configurations at their full BASELINE size, where the CPU oracle is
    too slow: size-independent properties of the degree sort (origin is a
    permutation, degrees ascend, every sorted row is its original row) and of
    the task list (tasks_check: every row covered, every nonzero owned once),
    and the aggregation at the configuration's S, values passed as NULL as
    bench.py passes them, against the float64 device reference over the
    UNSORTED CSR (no sort, partition or task code in common) on every row."""
    rowoff, col, val, X = graphs.build_config_torch(cfg, "cuda")
    n, nnz, K = rowoff.numel() - 1, col.numel(), X.shape[1]
    dev = X.device
    assert bool((val == 1.0).all())
    org = torch.empty(n, dtype=torch.int32, device=dev)
    sro = torch.empty(n + 1, dtype=torch.int32, device=dev)
    scol = torch.empty(nnz, dtype=torch.int32, device=dev)
    sval = torch.empty(nnz, dtype=torch.float32, device=dev)
    ctx.sort_by_degree_device(n, nnz, rowoff.data_ptr(), col.data_ptr(), val.data_ptr(),
                              org.data_ptr(), sro.data_ptr(), scol.data_ptr(), sval.data_ptr())
    torch.cuda.synchronize()
    o = org.long()
    assert torch.equal(torch.bincount(o, minlength=n), torch.ones(n, dtype=torch.long, device=dev))
    deg_sorted = (sro[1:] - sro[:-1]).long()
    deg_orig = (rowoff[1:] - rowoff[:-1]).long()
    assert bool((deg_sorted[1:] >= deg_sorted[:-1]).all())
    assert torch.equal(deg_sorted, deg_orig[o])
    # Each sorted row holds its original row's column ids, in order.
    starts = rowoff[:-1].long()[o]
    idx = torch.repeat_interleave(starts - sro[:-1].long(), deg_sorted) + \
        torch.arange(nnz, device=dev)
    assert torch.equal(scol, col[idx])
    del idx, starts

    costs = cs.read_costs_one_per_line(COSTS_FILE)
    S = graphs.CONFIGS[cfg]["S"]
    ptr, n_tasks = ctx.partition_device(n, sro.data_ptr(), costs, cs.capacity_from_s(S, costs))
    tasks = torch.as_tensor(_DevInt32(ptr, n_tasks * 4), device=dev).clone()
    torch.cuda.synchronize()
    chk = ctx.tasks_check(n, nnz, sro.data_ptr(), tasks.data_ptr(), n_tasks)
    assert chk == dict(bad_tasks=0, uncovered_rows=0, nnz_coverage_errors=0)

    out = torch.full((n, K), float("nan"), dtype=torch.float32, device=dev)
    ctx.spmm_mean_device(n, nnz, sro.data_ptr(), scol.data_ptr(), 0, org.data_ptr(),
                         X.data_ptr(), n, K, tasks.data_ptr(), n_tasks, out.data_ptr(),
                         cs.ROWS_COVERED)
    ref = torch.empty_like(out)
    ctx.spmm_mean_reference_device(n, nnz, rowoff.data_ptr(), col.data_ptr(), val.data_ptr(),
                                   X.data_ptr(), n, K, ref.data_ptr())
    torch.cuda.synchronize()
    assert ctx.take_device_errors() == 0
    X.abs_()
    scale = torch.empty_like(out)
    ctx.spmm_mean_reference_device(n, nnz, rowoff.data_ptr(), col.data_ptr(), val.data_ptr(),
                                   X.data_ptr(), n, K, scale.data_ptr())
    torch.cuda.synchronize()
    scale = torch.maximum(scale, ref.abs())
    err = torch.where(scale > 0, (out - ref).abs() / scale, (out - ref).abs())
    assert not bool(torch.isnan(out).any())
    worst = float(err.max())
    assert worst <= 1e-5, f"config {cfg}: max condition-relative error {worst:.3e}"
