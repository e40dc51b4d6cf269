"""GPU tests of aggregation plans (cwlb_plan_*) through the C ABI.

A plan must compute exactly the task list's aggregation (the reference's
spmmKernel semantics, src/parallelMatrix.cpp:151-236) whatever it decides:

  * grouped plans (unit values, column-sorted rows, hub rows split into
    fragments) against the oracle's float64 mean, within the condition-relative
    1e-5 of tests/helpers.py, for K = 32, 64 and 128, with and without
    CWLB_ROWS_COVERED, twice in a row on the same output buffer;
  * rows that one task covers whole: bit-identical to the task kernel's (they
    are never grouped);
  * the fallbacks (weighted values, unsorted rows, group size 1, K outside
    {32, 64, 128}, unaligned H, CWLB_DETERMINISTIC) report why and still
    match;
  * a task list that covers only part of the graph: only those nonzeros count;
  * a column outside H raises the device error flag instead of faulting.
"""
import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from helpers import assert_mean_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

COSTS = cs.SpmmCostParams(0.005513, 0.018253, 0.010677, 0.504722)
COSTS_L = [COSTS.C_compute_ns, COSTS.C_load_ns, COSTS.C_store_ns, COSTS.C_atomic_ns]


@pytest.fixture(scope="module")
def ctx():
    c = cs.Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def _sorted_graph(oracle, scale=13, edges=600_000, seed=51, values=None, shuffle_rows=False):
    ro, col, val = graphs.rmat_np(scale, edges, 0.57, 0.19, 0.19, seed=seed, symmetrize=True,
                                  drop_self_loops=True, dedupe=True)
    if values is not None:
        val = values(len(col))
    if shuffle_rows:
        rng = np.random.default_rng(seed)
        col = col.copy()
        for r in range(0, len(ro) - 1, 7):  # every 7th row's columns out of order
            rng.shuffle(col[ro[r]:ro[r + 1]])
    return oracle.sort_by_degree(ro, col, val)


class _Case:
    def __init__(self, ctx, oracle, origin, sro, scol, sval, S, K, tasks=None):
        self.ctx, self.oracle = ctx, oracle
        self.origin, self.sro, self.scol, self.sval = origin, sro, scol, sval
        self.n, self.nnz, self.K = len(origin), len(scol), K
        self.d = {k: torch.from_numpy(v).cuda() for k, v in
                  dict(org=origin, sro=sro, scol=scol, sval=sval).items()}
        self.tasks = oracle.partition(sro, COSTS_L, cs.capacity_from_s(S, COSTS)) \
            if tasks is None else tasks
        self.d_tasks = torch.from_numpy(np.ascontiguousarray(self.tasks, np.int32)).cuda()
        self.X = graphs.uniform_features_np(self.n, K, seed=52)
        self.d_X = torch.from_numpy(self.X).cuda()

    def plan(self, group_size=0):
        return cs.Plan(self.ctx, self.n, self.nnz, self.d["sro"].data_ptr(),
                       self.d["scol"].data_ptr(), self.d["sval"].data_ptr(),
                       self.d_tasks.data_ptr(), len(self.tasks), group_size)

    def run(self, plan, flags=0, out=None, X=None):
        X = self.d_X if X is None else X
        if out is None:
            out = torch.full((self.n, X.shape[1]), float("nan"), device="cuda")
        plan.aggregate_device(self.d["org"].data_ptr(), X.data_ptr(), X.shape[0], X.shape[1],
                              out.data_ptr(), flags)
        torch.cuda.synchronize()
        assert self.ctx.take_device_errors() == 0
        return out

    def check(self, out, what):
        ref, cond = self.oracle.spmm_mean_f64(self.sro, self.scol, self.sval, self.origin, self.X)
        assert_mean_close(out.cpu().numpy(), ref, cond, what=what)

    def whole_rows(self):
        """Original ids of the rows one task covers whole."""
        deg = np.diff(self.sro)
        rows = []
        for rs, re_, fo, ln in self.tasks:
            for r in range(rs, re_):
                b = fo if r == rs else 0
                e = ln if (r == re_ - 1 and ln > 0) else deg[r]
                if b == 0 and e == deg[r]:
                    rows.append(self.origin[r])
        return np.array(rows, np.int64)


@pytest.mark.parametrize("K", [128, 64, 32])
@pytest.mark.parametrize("gs", [8, 4])
def test_grouped_plan_matches_oracle(ctx, oracle, K, gs):
    case = _Case(ctx, oracle, *_sorted_graph(oracle), S=40, K=K)
    plan = case.plan(gs)
    info = plan.info()
    assert info["group_size"] == gs and info["off_reason"] == 0, info
    assert 0 < info["union_entries"] < info["grouped_nnz"]
    for flags in (0, cs.ROWS_COVERED):
        out = case.run(plan, flags)
        case.check(out, f"plan K={K} gs={gs} flags={flags}")
        out = case.run(plan, flags, out=out)  # again, into the previous result
        case.check(out, f"plan K={K} gs={gs} flags={flags}, second call")
    plan.close()


def test_plan_matches_the_task_kernel(ctx, oracle):
    case = _Case(ctx, oracle, *_sorted_graph(oracle, seed=53), S=64, K=128)
    plan = case.plan()
    assert plan.info()["group_size"] == 4  # the default
    out_p = case.run(plan, cs.ROWS_COVERED)
    out_t = torch.full_like(out_p, float("nan"))
    ctx.spmm_mean_device(case.n, case.nnz, case.d["sro"].data_ptr(), case.d["scol"].data_ptr(),
                         case.d["sval"].data_ptr(), case.d["org"].data_ptr(), case.d_X.data_ptr(),
                         case.n, 128, case.d_tasks.data_ptr(), len(case.tasks), out_t.data_ptr(),
                         cs.ROWS_COVERED)
    torch.cuda.synchronize()
    # Rows one task covers whole are never grouped: the same kernel computes
    # them in the same order, so they are bit-identical.
    whole = case.whole_rows()
    assert len(whole) > 0
    a, b = out_p.cpu().numpy(), out_t.cpu().numpy()
    assert np.array_equal(a[whole].view(np.uint32), b[whole].view(np.uint32))
    case.check(out_p, "plan vs oracle")
    plan.close()


@pytest.mark.parametrize("kind,reason", [
    ("weighted", cs.PLAN_VALUES),
    ("unsorted", cs.PLAN_UNSORTED),
    ("disabled", cs.PLAN_DISABLED),
])
def test_plan_fallbacks_report_why_and_match(ctx, oracle, kind, reason):
    if kind == "weighted":
        g = _sorted_graph(oracle, values=lambda m: np.random.default_rng(5).uniform(
            0.5, 1.5, m).astype(np.float32))
    elif kind == "unsorted":
        g = _sorted_graph(oracle, shuffle_rows=True)
    else:
        g = _sorted_graph(oracle)
    case = _Case(ctx, oracle, *g, S=40, K=64)
    plan = case.plan(1 if kind == "disabled" else 0)
    info = plan.info()
    assert info["group_size"] == 0 and info["off_reason"] & reason, info
    out = case.run(plan, cs.ROWS_COVERED)
    case.check(out, f"fallback {kind}")
    plan.close()


def test_plan_per_call_fallbacks_match(ctx, oracle):
    case = _Case(ctx, oracle, *_sorted_graph(oracle, seed=54), S=40, K=96)
    plan = case.plan()
    assert plan.info()["group_size"] == 4  # built; K = 96 runs the task kernel
    case.check(case.run(plan, cs.ROWS_COVERED), "K=96")
    # Deterministic merge: the task kernel's fixed order, bit-identical twice.
    a = case.run(plan, cs.ROWS_COVERED | cs.DETERMINISTIC).cpu().numpy()
    b = case.run(plan, cs.ROWS_COVERED | cs.DETERMINISTIC).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # Unaligned H (a view starting one float in) takes the task kernel too.
    Xb = torch.zeros(case.n * 96 + 1, device="cuda")
    Xb[1:] = case.d_X.reshape(-1)
    Xv = Xb[1:].view(case.n, 96)
    case.check(case.run(plan, cs.ROWS_COVERED, X=Xv), "unaligned H")
    plan.close()


def test_plan_honours_a_partial_task_list(ctx, oracle):
    origin, sro, scol, sval = _sorted_graph(oracle, seed=55)
    tasks = oracle.partition(sro, COSTS_L, cs.capacity_from_s(40, COSTS))
    part = np.ascontiguousarray(tasks[::3])  # every third task only
    case = _Case(ctx, oracle, origin, sro, scol, sval, S=40, K=128, tasks=part)
    plan = case.plan()
    assert plan.info()["group_size"] == 4  # the default
    out = case.run(plan, 0)
    want = oracle.spmm_mean(sro, scol, sval, origin, case.X, part)
    err = np.abs(out.cpu().numpy() - want).max()
    assert err <= 1e-5 * max(1.0, np.abs(want).max())
    plan.close()


def test_plan_column_outside_h_raises_the_device_flag(ctx, oracle):
    case = _Case(ctx, oracle, *_sorted_graph(oracle, seed=56), S=40, K=64)
    plan = case.plan()
    assert plan.info()["group_size"] == 4  # the default
    short = case.d_X[: case.n // 2].contiguous()  # H without its upper half
    out = torch.zeros((case.n, 64), device="cuda")
    plan.aggregate_device(case.d["org"].data_ptr(), short.data_ptr(), short.shape[0], 64,
                          out.data_ptr(), cs.ROWS_COVERED)
    torch.cuda.synchronize()
    assert ctx.take_device_errors() & cs.DEVERR_COL_RANGE
    plan.close()
