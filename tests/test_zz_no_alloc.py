"""The partitioner entry point that allocates no device memory.

cwlb_partition_device_noalloc serves callers that cannot let a library call
cudaMalloc/cudaFree (their device memory belongs to another allocator, or a
pool sized once at start-up) and that would not want those calls to
synchronise the device mid-pipeline.  It keeps its scratch in one fixed
8 MiB device array and writes into the caller's task buffer.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.  It must pass both alone in a
fresh process and after the rest of the suite.  The checks call the new entry
point through the C ABI and compare its task list, bit for bit (the tolerance
of every partition test), with the existing entry point cwlb_partition_device,
on two calls in a row whose inputs differ (so stale scratch from the first
call cannot leak into the second).
"""
import ctypes as C

import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from helpers import sorted_rowoff_from_degrees

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

_noalloc = cs._lib.cwlb_partition_device_noalloc
_noalloc.argtypes = [C.c_void_p, C.c_int32, C.c_void_p, C.POINTER(cs.cwlb_costs), C.c_double,
                     C.c_void_p, C.c_int64, C.POINTER(C.c_int64)]
_noalloc.restype = C.c_int

MAX_ROWS = 1048576  # CWLB_NOALLOC_MAX_ROWS in include/cwlb_spmm.h


class _DevInt32:
    def __init__(self, ptr, count):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3}


@pytest.fixture(scope="module")
def ctx():
    c = cs.Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def _call_noalloc(d_rowoff, n_rows, costs, cap, out, max_tasks):
    n = C.c_int64(-1)
    c = costs.c()
    rc = _noalloc(C.c_void_p(torch.cuda.current_stream().cuda_stream), n_rows,
                  d_rowoff.data_ptr(), C.byref(c), float(cap),
                  out.data_ptr() if out is not None else None, max_tasks, C.byref(n))
    return rc, n.value


def _existing_entry_point(ctx, d_rowoff, n_rows, costs, cap):
    ptr, cnt = ctx.partition_device(n_rows, d_rowoff.data_ptr(), costs, cap)
    if cnt == 0:
        return np.zeros((0, 4), np.int32)
    t = torch.as_tensor(_DevInt32(ptr, cnt * 4), device="cuda").clone()
    torch.cuda.synchronize()
    return t.view(cnt, 4).cpu().numpy()


def _cases():
    ro_a, col_a, val_a = graphs.rmat_np(14, 300_000, 0.57, 0.19, 0.19, seed=21, symmetrize=True,
                                        drop_self_loops=True, dedupe=True)
    deg_a = np.sort(np.diff(ro_a))
    rng = np.random.default_rng(22)
    deg_b = np.minimum((rng.pareto(1.1, 3000) * 5).astype(np.int64), 20000)
    return [
        (sorted_rowoff_from_degrees(deg_a), cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5), 24),
        (sorted_rowoff_from_degrees(deg_b), cs.SpmmCostParams(1.0, 2.0, 0.5, 3.0), 7),
    ]


def test_noalloc_matches_existing_entry_point_on_two_calls_in_a_row(ctx):
    cases = _cases()
    # Set-up: the first call on the device looks up the scratch address.
    ro0, costs0, S0 = cases[0]
    d0 = torch.from_numpy(ro0).cuda()
    probe = torch.empty((1, 4), dtype=torch.int32, device="cuda")
    _call_noalloc(d0, len(ro0) - 1, costs0, cs.capacity_from_s(S0, costs0), probe, 0)
    torch.cuda.synchronize()
    for ro, costs, S in cases:
        n_rows = len(ro) - 1
        d_ro = torch.from_numpy(ro).cuda()
        cap = cs.capacity_from_s(S, costs)
        want = _existing_entry_point(ctx, d_ro, n_rows, costs, cap)
        out = torch.full((len(want) + 8, 4), -7, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc, n = _call_noalloc(d_ro, n_rows, costs, cap, out, out.shape[0])
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        assert rc == cs.OK, cs._lib.cwlb_last_error().decode()
        assert n == len(want)
        got = out[:n].cpu().numpy()
        assert np.array_equal(got, want)
        assert (out[n:].cpu().numpy() == -7).all()  # nothing written past the task list
        assert free_after == free_before  # no device allocation happened


def test_noalloc_literal_path_matches(ctx):
    # Non-finite costs take the literal restatement; same answer either way.
    ro = sorted_rowoff_from_degrees(np.concatenate([np.zeros(40, int), np.arange(1, 300) % 90]))
    costs = cs.SpmmCostParams(float("nan"), 1.0, 0.5, 2.0)
    d_ro = torch.from_numpy(ro).cuda()
    want = _existing_entry_point(ctx, d_ro, len(ro) - 1, costs, 40.0)
    out = torch.empty((len(want) + 1, 4), dtype=torch.int32, device="cuda")
    rc, n = _call_noalloc(d_ro, len(ro) - 1, costs, 40.0, out, out.shape[0])
    torch.cuda.synchronize()
    assert rc == cs.OK and n == len(want)
    assert np.array_equal(out[:n].cpu().numpy(), want)


def test_noalloc_rejects_sizes_beyond_its_limits():
    tiny = torch.zeros(2, dtype=torch.int32, device="cuda")
    costs = cs.SpmmCostParams(0.1, 0.2, 0.3, 0.4)
    rc, _ = _call_noalloc(tiny, MAX_ROWS + 1, costs, 10.0, None, 0)
    assert rc == cs.ERR_INVALID_ARGUMENT
    assert "no-allocation scratch limit" in cs._lib.cwlb_last_error().decode()
    ro = sorted_rowoff_from_degrees(np.arange(40))
    d_ro = torch.from_numpy(ro).cuda()
    out = torch.empty((2, 4), dtype=torch.int32, device="cuda")
    rc, n = _call_noalloc(d_ro, 40, costs, cs.capacity_from_s(4, costs), out, 2)
    assert rc == cs.ERR_BUFFER_TOO_SMALL and n > 2


def test_noalloc_rejects_a_null_task_buffer_before_any_launch():
    # Host-side check only: a NULL buffer with a positive capacity is refused
    # before the call looks up its scratch or launches a kernel.
    ro = sorted_rowoff_from_degrees(np.arange(40))
    d_ro = torch.from_numpy(ro).cuda()
    costs = cs.SpmmCostParams(0.1, 0.2, 0.3, 0.4)
    rc, n = _call_noalloc(d_ro, 40, costs, cs.capacity_from_s(4, costs), None, 5)
    assert rc == cs.ERR_INVALID_ARGUMENT
    assert "null argument" in cs._lib.cwlb_last_error().decode()
    assert n == -1  # the count is not written on a rejected call


def test_noalloc_rejects_more_distinct_degrees_than_its_run_limit():
    # Degrees 0..16384 give 16385 runs of equal degree, one more than the
    # scratch holds.  Only the offsets are read, so nnz (1.3e8) costs nothing.
    max_runs = 16384  # CWLB_NOALLOC_MAX_RUNS in include/cwlb_spmm.h
    ro = sorted_rowoff_from_degrees(np.arange(max_runs + 1))
    d_ro = torch.from_numpy(ro).cuda()
    costs = cs.SpmmCostParams(0.1, 0.2, 0.3, 0.4)
    out = torch.full((64, 4), -7, dtype=torch.int32, device="cuda")
    rc, _ = _call_noalloc(d_ro, len(ro) - 1, costs, cs.capacity_from_s(32, costs), out, 64)
    torch.cuda.synchronize()
    assert rc == cs.ERR_INVALID_ARGUMENT
    assert "distinct row degrees" in cs._lib.cwlb_last_error().decode()
    assert (out.cpu().numpy() == -7).all()  # the task buffer is untouched
