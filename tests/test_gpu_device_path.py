"""GPU: the device-resident pipeline (sort -> partition -> aggregate) that the
benchmark times, driven through the C ABI with torch-allocated buffers."""
import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from helpers import assert_mean_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    c = cs.Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def _device_pipeline(ctx, rowoff, col, val, X, costs, S):
    dev = torch.device("cuda:0")
    n, nnz = len(rowoff) - 1, len(col)
    d_ro = torch.from_numpy(rowoff).to(dev)
    d_col = torch.from_numpy(col).to(dev)
    d_val = torch.from_numpy(val).to(dev)
    d_X = torch.from_numpy(X).to(dev)
    org = torch.empty(n, dtype=torch.int32, device=dev)
    sro = torch.empty(n + 1, dtype=torch.int32, device=dev)
    scol = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    sval = torch.empty(max(nnz, 1), dtype=torch.float32, device=dev)
    ctx.sort_by_degree_device(n, nnz, d_ro.data_ptr(), d_col.data_ptr(), d_val.data_ptr(),
                              org.data_ptr(), sro.data_ptr(), scol.data_ptr(), sval.data_ptr())
    cap = cs.capacity_from_s(S, costs)
    t_ptr, n_tasks = ctx.partition_device(n, sro.data_ptr(), costs, cap)
    return dict(org=org, sro=sro, scol=scol, sval=sval, X=d_X, t_ptr=t_ptr, n_tasks=n_tasks,
                cap=cap, n=n, nnz=nnz)


def test_device_pipeline_matches_oracle(ctx, oracle):
    rowoff, col, val = graphs.rmat_np(14, 400_000, 0.57, 0.19, 0.19, seed=9, symmetrize=True,
                                      drop_self_loops=True, dedupe=True)
    n = len(rowoff) - 1
    K = 64
    X = graphs.uniform_features_np(n, K, seed=9)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    p = _device_pipeline(ctx, rowoff, col, val, X, costs, 24)
    o = oracle.sort_by_degree(rowoff, col, val)
    assert np.array_equal(p["org"].cpu().numpy(), o[0])
    assert np.array_equal(p["sro"].cpu().numpy(), o[1])
    assert np.array_equal(p["scol"][:p["nnz"]].cpu().numpy(), o[2])
    want = oracle.partition(o[1], [0.02, 0.7, 0.3, 0.5], p["cap"])
    torch.cuda.synchronize()
    chk = ctx.tasks_check(n, p["nnz"], p["sro"].data_ptr(), p["t_ptr"], p["n_tasks"])
    assert chk == dict(bad_tasks=0, uncovered_rows=0, nnz_coverage_errors=0)
    out_full = torch.empty((n, K), dtype=torch.float32, device="cuda:0")
    out_cov = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda:0")
    args = (n, p["nnz"], p["sro"].data_ptr(), p["scol"].data_ptr(), p["sval"].data_ptr(),
            p["org"].data_ptr(), p["X"].data_ptr(), n, K, p["t_ptr"], p["n_tasks"])
    ctx.spmm_mean_device(*args, out_full.data_ptr(), 0)
    ctx.spmm_mean_device(*args, out_cov.data_ptr(), cs.ROWS_COVERED)
    torch.cuda.synchronize()
    assert ctx.take_device_errors() == 0
    ref, cond = oracle.spmm_mean_f64(o[1], o[2], o[3], o[0], X)
    assert_mean_close(out_full.cpu().numpy(), ref, cond, what="device pipeline")
    assert_mean_close(out_cov.cpu().numpy(), ref, cond, what="rows-covered mode")
    # the task list itself, copied back through a host-buffer partition call
    host_tasks = ctx.costWeightedTaskPartitioning(cs.CSR(o[1], o[2], o[3]), costs, p["cap"])
    assert np.array_equal(host_tasks, want)
    assert len(want) == p["n_tasks"]


def test_tasks_check_detects_gaps(ctx):
    rowoff = np.array([0, 2, 4, 4, 7], np.int32)
    d_ro = torch.from_numpy(rowoff).cuda()
    good = torch.tensor([[0, 2, 0, 0], [2, 4, 0, 0]], dtype=torch.int32, device="cuda:0")
    gap = torch.tensor([[0, 1, 0, 0], [3, 4, 1, 0]], dtype=torch.int32, device="cuda:0")
    bad = torch.tensor([[0, 9, 0, 0]], dtype=torch.int32, device="cuda:0")
    assert ctx.tasks_check(4, 7, d_ro.data_ptr(), good.data_ptr(), 2) == dict(
        bad_tasks=0, uncovered_rows=0, nnz_coverage_errors=0)
    r = ctx.tasks_check(4, 7, d_ro.data_ptr(), gap.data_ptr(), 2)
    assert r["uncovered_rows"] == 2 and r["nnz_coverage_errors"] == 3
    assert ctx.tasks_check(4, 7, d_ro.data_ptr(), bad.data_ptr(), 1)["bad_tasks"] == 1


def _aggregate_vs_torch(ctx, n, h_rows, K, deg, col, val, X, S=64):
    """Sort, partition and aggregate on the device through the C ABI; compare
    with a float64 reference computed by torch on the device."""
    dev = X.device
    rowoff = torch.zeros(n + 1, dtype=torch.int64, device=dev)
    rowoff[1:] = torch.cumsum(deg, 0)
    nnz = int(rowoff[-1])
    ro32 = rowoff.to(torch.int32)
    org = torch.empty(n, dtype=torch.int32, device=dev)
    sro = torch.empty(n + 1, dtype=torch.int32, device=dev)
    scol = torch.empty(nnz, dtype=torch.int32, device=dev)
    sval = torch.empty(nnz, dtype=torch.float32, device=dev)
    ctx.sort_by_degree_device(n, nnz, ro32.data_ptr(), col.data_ptr(), val.data_ptr(),
                              org.data_ptr(), sro.data_ptr(), scol.data_ptr(), sval.data_ptr())
    costs = cs.SpmmCostParams(0.0055, 0.018, 0.011, 0.5)
    t_ptr, n_tasks = ctx.partition_device(n, sro.data_ptr(), costs, cs.capacity_from_s(S, costs))
    out = torch.full((n, K), float("nan"), device=dev)
    ctx.spmm_mean_device(n, nnz, sro.data_ptr(), scol.data_ptr(), sval.data_ptr(), org.data_ptr(),
                         X.data_ptr(), h_rows, K, t_ptr, n_tasks, out.data_ptr(), 0)
    torch.cuda.synchronize()
    assert ctx.take_device_errors() == 0
    rows = torch.repeat_interleave(torch.arange(n, device=dev), deg)
    ref = torch.zeros((n, K), dtype=torch.float64, device=dev)
    cond = torch.zeros((n, K), dtype=torch.float64, device=dev)
    for c0 in range(0, nnz, 200_000):
        c1 = min(nnz, c0 + 200_000)
        prod = X[col[c0:c1].long()].double() * val[c0:c1].double()[:, None]
        ref.index_add_(0, rows[c0:c1], prod)
        cond.index_add_(0, rows[c0:c1], prod.abs())
    d = deg.clamp_min(1).double()[:, None]
    ref /= d
    cond /= d
    err = (out.double() - ref).abs()
    scale = torch.maximum(ref.abs(), cond)
    bad = err > 1e-5 * scale
    bad &= ~((scale == 0) & (err == 0))
    assert int(bad.sum()) == 0, float((err / scale.clamp_min(1e-30)).max())


def test_x_far_larger_than_l2(ctx):
    """X of 2.3M x 256 floats (2.4 GB, far larger than L2; most gathers miss
    L2), checked against a float64 reference computed on the device by torch."""
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    n, h_rows, K = 20000, 2_300_000, 256
    deg = torch.randint(0, 60, (n,), generator=g, device=dev)
    deg[::997] = 700  # a few long rows (split into fragments)
    nnz = int(deg.sum())
    col = torch.randint(0, h_rows, (nnz,), generator=g, device=dev, dtype=torch.int32)
    val = torch.randn(nnz, generator=g, device=dev)
    X = torch.randn((h_rows, K), generator=g, device=dev)
    _aggregate_vs_torch(ctx, n, h_rows, K, deg, col, val, X)


@pytest.mark.parametrize("K", [256, 254])
def test_x_beyond_2_pow_31_elements(ctx, K):
    """X with more than 2^31 elements (8.6M x K floats, 8.8 GB), half of the
    gathers aimed at its last 100K rows: element offsets past 2^31 must be
    formed in 64 bits, in the float4 kernel (K = 256) and in the scalar one
    (K = 254)."""
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(K)
    n, h_rows = 5000, 8_600_000
    assert h_rows * K > 2 ** 31
    deg = torch.randint(0, 40, (n,), generator=g, device=dev)
    deg[::499] = 400
    nnz = int(deg.sum())
    col = torch.randint(0, h_rows, (nnz,), generator=g, device=dev, dtype=torch.int32)
    top = torch.randint(h_rows - 100_000, h_rows, (nnz,), generator=g, device=dev,
                        dtype=torch.int32)
    col = torch.where(torch.rand(nnz, generator=g, device=dev) < 0.5, top, col)
    val = torch.randn(nnz, generator=g, device=dev)
    X = torch.randn((h_rows, K), generator=g, device=dev)
    _aggregate_vs_torch(ctx, n, h_rows, K, deg, col, val, X)
    del X
    torch.cuda.empty_cache()


@pytest.mark.parametrize("K", [1, 7, 32, 300])
def test_reference_kernel_matches_oracle_f64(ctx, oracle, K):
    """cwlb_spmm_mean_reference_device (unsorted CSR, float64 sums, one
    rounding) against the oracle's exact mean: within one float rounding."""
    rng = np.random.default_rng(40 + K)
    from helpers import random_csr
    rowoff, col, val = random_csr(rng, 3000, 40, n_cols=2500, hubs=3, hub_factor=200)
    n, nnz = len(rowoff) - 1, len(col)
    X = rng.standard_normal((2500, K)).astype(np.float32)
    dev = torch.device("cuda:0")
    d = [torch.from_numpy(a).to(dev) for a in (rowoff, col, val, X)]
    out = torch.full((n, K), float("nan"), device=dev)
    ctx.spmm_mean_reference_device(n, nnz, d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(),
                                   d[3].data_ptr(), 2500, K, out.data_ptr())
    torch.cuda.synchronize()
    assert ctx.take_device_errors() == 0
    ref, cond = oracle.spmm_mean_f64(rowoff, col, val, np.arange(n, dtype=np.int32), X)
    got = out.cpu().numpy().astype(np.float64)
    # Rounded once from a double sum: error <= half an ulp of the result plus
    # the two double sums' own errors (below 1e-11 of the condition scale for
    # rows of up to 8000 nonzeros).
    scale = np.maximum(np.abs(ref), cond)
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -24 + 1e-11 * scale)
    assert np.all(got[np.diff(rowoff) == 0] == 0.0)


def test_reference_kernel_flags_bad_columns(ctx):
    dev = torch.device("cuda:0")
    ro = torch.tensor([0, 2, 3], dtype=torch.int32, device=dev)
    col = torch.tensor([0, 5, 1], dtype=torch.int32, device=dev)  # 5 >= h_rows
    val = torch.ones(3, device=dev)
    X = torch.arange(8, dtype=torch.float32, device=dev).reshape(2, 4)
    out = torch.empty((2, 4), device=dev)
    ctx.spmm_mean_reference_device(2, 3, ro.data_ptr(), col.data_ptr(), val.data_ptr(),
                                   X.data_ptr(), 2, 4, out.data_ptr())
    torch.cuda.synchronize()
    assert ctx.take_device_errors() == cs.DEVERR_COL_RANGE
    # The bad entry is skipped; the mean still divides by the stored degree.
    assert torch.equal(out.cpu(), torch.tensor([[0., 0.5, 1., 1.5], [4., 5., 6., 7.]]))


@pytest.mark.parametrize("K,S,covered", [(7, 16, False), (32, 16, True), (128, 9, True),
                                         (512, 64, False), (1100, 32, True)])
def test_deterministic_mode_is_reproducible(ctx, oracle, K, S, covered):
    """CWLB_DETERMINISTIC merges split rows in task order: two runs give the
    same bits, the result is within the tolerance of the exact mean, and rows
    that are never split equal the atomic mode's."""
    rng = np.random.default_rng(300 + K)
    from helpers import random_csr
    rowoff, col, val = random_csr(rng, 4000, 80, n_cols=3000, hubs=4, hub_factor=60)
    X = rng.standard_normal((3000, K)).astype(np.float32)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    p = _device_pipeline(ctx, rowoff, col, val, X, costs, S)
    n = p["n"]
    flags = cs.DETERMINISTIC | (cs.ROWS_COVERED if covered else 0)
    outs = []
    for f in (flags, flags, cs.ROWS_COVERED if covered else 0):
        out = torch.full((n, K), float("nan"), device="cuda:0")
        if not covered:
            out.zero_()
        ctx.spmm_mean_device(n, p["nnz"], p["sro"].data_ptr(), p["scol"].data_ptr(),
                             p["sval"].data_ptr(), p["org"].data_ptr(), p["X"].data_ptr(), 3000, K,
                             p["t_ptr"], p["n_tasks"], out.data_ptr(), f)
        torch.cuda.synchronize()
        assert ctx.take_device_errors() == 0
        outs.append(out.cpu().numpy())
    det1, det2, atomic = outs
    assert np.array_equal(det1, det2)
    o = oracle.sort_by_degree(rowoff, col, val)
    ref, cond = oracle.spmm_mean_f64(o[1], o[2], o[3], o[0], X)
    assert_mean_close(det1, ref, cond, what=f"deterministic K={K}")
    tasks = torch.as_tensor(_DevTasks(p["t_ptr"], p["n_tasks"]), device="cuda:0").cpu().numpy()
    tasks = tasks.reshape(-1, 4)
    deg = np.diff(o[1])
    split = set()
    for rs, re_, fo, ln in tasks:
        for r in (rs, re_ - 1):
            b = fo if r == rs else 0
            e = ln if (r == re_ - 1 and ln > 0) else deg[r]
            if deg[r] > 0 and b < e and not (b == 0 and e == deg[r]):
                split.add(int(r))
    assert split, "the case must split rows"
    keep = np.ones(n, bool)
    keep[o[0][sorted(split)]] = False
    assert np.array_equal(det1[keep], atomic[keep])


class _DevTasks:
    def __init__(self, ptr, count):
        self.__cuda_array_interface__ = {"shape": (count * 4,), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3}


@pytest.mark.parametrize("row_floats", [32, 128, 512])
def test_gather_rate_microbenchmark(ctx, row_floats):
    """The ceilings the bench reports: random rows gathered from a buffer that
    fits in L2 arrive faster than from one far larger than L2 (HBM), and both
    rates are plausible for a B200."""
    l2 = ctx.measure_gather_gbs(48, row_floats, 5)
    hbm = ctx.measure_gather_gbs(4096, row_floats, 5)
    assert 500.0 < hbm < 10000.0, hbm
    assert l2 > 1.5 * hbm, (l2, hbm)


@pytest.mark.parametrize("args", [(0, 128, 1), (48, 0, 1), (48, 12, 1), (48, 2048, 1), (48, 128, 0)])
def test_gather_rate_microbenchmark_rejects_bad_arguments(ctx, args):
    with pytest.raises(ValueError):
        ctx.measure_gather_gbs(*args)


@pytest.mark.parametrize("K,S", [(7, 24), (32, 220), (32, 16), (64, 40), (128, 40), (512, 40),
                                 (1100, 40)])
def test_null_values_equal_an_array_of_ones_bit_for_bit(ctx, oracle, K, S):
    """d_value == NULL means every value is 1.0: the kernels then load and
    broadcast no values, and fma(1, x, acc) rounds exactly as the general
    kernel's, so with the merge order fixed (CWLB_DETERMINISTIC) the output
    is bit-identical to passing an array of ones; with atomics, within the
    tolerance.  S = 220 at K = 32 gives many rows per task (the short-row
    instance).  An out-of-range column raises the device flag either way."""
    rowoff, col, _ = graphs.rmat_np(13, 150_000, 0.57, 0.19, 0.19, seed=31, symmetrize=True,
                                    drop_self_loops=True, dedupe=True)
    n, nnz = len(rowoff) - 1, len(col)
    ones = np.ones(nnz, np.float32)
    X = graphs.uniform_features_np(n, K, seed=32)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    p = _device_pipeline(ctx, rowoff, col, ones, X, costs, S)
    torch.cuda.synchronize()

    def run(vals, flags, col_ptr=None):
        out = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda:0")
        ctx.spmm_mean_device(n, nnz, p["sro"].data_ptr(),
                             p["scol"].data_ptr() if col_ptr is None else col_ptr, vals,
                             p["org"].data_ptr(), p["X"].data_ptr(), n, K, p["t_ptr"],
                             p["n_tasks"], out.data_ptr(), flags)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    det = [run(v, cs.DETERMINISTIC) for v in (p["sval"].data_ptr(), 0)]
    assert ctx.take_device_errors() == 0
    assert np.array_equal(det[0].view(np.uint32), det[1].view(np.uint32))
    ref, cond = oracle.spmm_mean_f64(*[t.cpu().numpy() for t in (p["sro"], p["scol"][:nnz])],
                                     ones, p["org"].cpu().numpy(), X)
    assert_mean_close(run(0, 0), ref, cond, what=f"unit values K={K}, atomics")
    assert ctx.take_device_errors() == 0
    bad_col = p["scol"].clone()
    bad_col[int(p["sro"][-2]) + 3] = n + 5  # inside the largest row
    for vals in (p["sval"].data_ptr(), 0):
        run(vals, 0, bad_col.data_ptr())
        assert ctx.take_device_errors() & cs.DEVERR_COL_RANGE


@pytest.mark.parametrize("K,S", [(32, 512), (64, 1024), (128, 512), (512, 1024), (1100, 2048)])
def test_cta_per_task_variant_matches_oracle(ctx, oracle, K, S):
    """A task list of at most 8 tasks per SM runs one CTA per task
    (spmm_cta_kernel: a hub fragment split over the CTA's eight warps and
    reduced through shared memory in warp order, the rows of a multi-row task
    spread over the warps).  Checked against the oracle with weighted and
    NULL (unit) values, with and without CWLB_ROWS_COVERED; in deterministic
    mode two runs are bit-identical and NULL values equal an array of ones."""
    rowoff, col, _ = graphs.rmat_np(13, 150_000, 0.57, 0.19, 0.19, seed=33, symmetrize=True,
                                    drop_self_loops=True, dedupe=True)
    n, nnz = len(rowoff) - 1, len(col)
    rng = np.random.default_rng(34)
    X = graphs.uniform_features_np(n, K, seed=35)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    sms = ctx.device_info()["max_compute_units"]
    for kind in ("weighted", "unit"):
        val = (rng.uniform(0.5, 1.5, nnz).astype(np.float32) if kind == "weighted"
               else np.ones(nnz, np.float32))
        p = _device_pipeline(ctx, rowoff, col, val, X, costs, S)
        torch.cuda.synchronize()
        assert 0 < p["n_tasks"] <= 8 * sms, p["n_tasks"]
        chk = ctx.tasks_check(n, nnz, p["sro"].data_ptr(), p["t_ptr"], p["n_tasks"])
        assert chk == dict(bad_tasks=0, uncovered_rows=0, nnz_coverage_errors=0)
        vptr = p["sval"].data_ptr() if kind == "weighted" else 0

        def run(flags, vals=vptr):
            out = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda:0")
            if not flags & cs.ROWS_COVERED:
                out.zero_()
            ctx.spmm_mean_device(n, nnz, p["sro"].data_ptr(), p["scol"].data_ptr(), vals,
                                 p["org"].data_ptr(), p["X"].data_ptr(), n, K, p["t_ptr"],
                                 p["n_tasks"], out.data_ptr(), flags)
            torch.cuda.synchronize()
            assert ctx.take_device_errors() == 0
            return out.cpu().numpy()

        ref, cond = oracle.spmm_mean_f64(p["sro"].cpu().numpy(), p["scol"][:nnz].cpu().numpy(),
                                         p["sval"][:nnz].cpu().numpy(), p["org"].cpu().numpy(), X)
        for flags in (0, cs.ROWS_COVERED):
            assert_mean_close(run(flags), ref, cond, what=f"CTA per task, {kind}, K={K}, {flags}")
        d1, d2 = run(cs.DETERMINISTIC), run(cs.DETERMINISTIC)
        assert np.array_equal(d1.view(np.uint32), d2.view(np.uint32))
        assert_mean_close(d1, ref, cond, what=f"CTA per task, {kind}, K={K}, deterministic")
        if kind == "unit":
            ones = run(cs.DETERMINISTIC, p["sval"].data_ptr())
            assert np.array_equal(d1.view(np.uint32), ones.view(np.uint32))


@pytest.mark.parametrize("K", [4, 32, 64, 100, 128, 512, 1100])
@pytest.mark.parametrize("graph", ["short_rows", "hubs"])
def test_task_variants_agree(ctx, oracle, K, graph):
    """The same task list through both kernel variants, forced with
    CWLB_TASK_PER_WARP / CWLB_TASK_PER_CTA: both within the tolerance of the
    oracle's float64 mean, and every whole row of a task of at least 32 rows
    (one lane group per row in both, nonzero order) bit-identical between
    them.  The short-row graph (~100 rows of degree ~4 per task) runs the
    warp variant's short-row instance."""
    from helpers import random_csr
    rng = np.random.default_rng(500 + K)
    if graph == "short_rows":
        d = rng.integers(1, 8, 20_000)
        rowoff = np.zeros(len(d) + 1, np.int32)
        rowoff[1:] = np.cumsum(d)
        col = rng.integers(0, 20_000, int(rowoff[-1])).astype(np.int32)
        val = rng.uniform(0.5, 1.5, len(col)).astype(np.float32)
        n_cols, S = 20_000, 300
    else:
        rowoff, col, val = random_csr(rng, 5000, 60, n_cols=4000, hubs=6, hub_factor=80)
        n_cols, S = 4000, 48
    n, nnz = len(rowoff) - 1, len(col)
    X = rng.standard_normal((n_cols, K)).astype(np.float32)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    p = _device_pipeline(ctx, rowoff, col, val, X, costs, S)
    torch.cuda.synchronize()

    def run(flags):
        out = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda:0")
        ctx.spmm_mean_device(n, nnz, p["sro"].data_ptr(), p["scol"].data_ptr(),
                             p["sval"].data_ptr(), p["org"].data_ptr(), p["X"].data_ptr(), n_cols,
                             K, p["t_ptr"], p["n_tasks"], out.data_ptr(),
                             cs.ROWS_COVERED | flags)
        torch.cuda.synchronize()
        assert ctx.take_device_errors() == 0
        return out.cpu().numpy()

    warp, cta = run(cs.TASK_PER_WARP), run(cs.TASK_PER_CTA)
    o = [t.cpu().numpy() for t in (p["sro"], p["scol"][:nnz], p["sval"][:nnz], p["org"])]
    ref, cond = oracle.spmm_mean_f64(o[0], o[1], o[2], o[3], X)
    assert_mean_close(warp, ref, cond, what=f"warp per task, K={K}, {graph}")
    assert_mean_close(cta, ref, cond, what=f"CTA per task, K={K}, {graph}")
    tasks = torch.as_tensor(_DevTasks(p["t_ptr"], p["n_tasks"]), device="cuda:0").cpu().numpy()
    deg = np.diff(o[0])
    rows = []
    for rs, re_, fo, ln in tasks.reshape(-1, 4):
        if re_ - rs < 32:
            continue
        for r in range(rs, re_):
            b = fo if r == rs else 0
            e = ln if (r == re_ - 1 and ln > 0) else deg[r]
            if b == 0 and e == deg[r]:
                rows.append(o[3][r])
    if graph == "short_rows":
        assert len(rows) > n // 2
    rows = np.array(rows, np.int64)
    assert np.array_equal(warp[rows].view(np.uint32), cta[rows].view(np.uint32))
    with pytest.raises(ValueError):
        run(cs.TASK_PER_WARP | cs.TASK_PER_CTA)
    with pytest.raises(ValueError):
        run(1 << 30)


@pytest.mark.parametrize("K,S", [(32, 8), (64, 16), (128, 32), (512, 16), (1100, 64)])
def test_task_runs_match_one_warp_per_task(ctx, oracle, K, S):
    """Small tasks (fewer than 128 nonzeros on average, a long list) run as
    warp runs of consecutive tasks (spmm_run_kernel): consecutive fragments of
    one row are summed in registers and written once.  Against the same list
    forced to one warp per task (CWLB_TASK_PER_WARP): both within the
    tolerance of the oracle's float64 mean, and every row one task covers
    whole bit-identical between them."""
    rowoff, col, _ = graphs.rmat_np(15, 1_200_000, 0.6, 0.15, 0.15, seed=37, symmetrize=True,
                                    drop_self_loops=True, dedupe=True)
    n, nnz = len(rowoff) - 1, len(col)
    rng = np.random.default_rng(38)
    val = rng.uniform(0.5, 1.5, nnz).astype(np.float32)
    X = graphs.uniform_features_np(n, K, seed=39)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    p = _device_pipeline(ctx, rowoff, col, val, X, costs, S)
    torch.cuda.synchronize()
    sms = ctx.device_info()["max_compute_units"]
    assert p["n_tasks"] > 128 * sms and nnz / p["n_tasks"] < 128 and n < 16 * p["n_tasks"]

    def run(flags):
        out = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda:0")
        ctx.spmm_mean_device(n, nnz, p["sro"].data_ptr(), p["scol"].data_ptr(),
                             p["sval"].data_ptr(), p["org"].data_ptr(), p["X"].data_ptr(), n, K,
                             p["t_ptr"], p["n_tasks"], out.data_ptr(), cs.ROWS_COVERED | flags)
        torch.cuda.synchronize()
        assert ctx.take_device_errors() == 0
        return out.cpu().numpy()

    runs, warp = run(0), run(cs.TASK_PER_WARP)
    o = [t.cpu().numpy() for t in (p["sro"], p["scol"][:nnz], p["sval"][:nnz], p["org"])]
    ref, cond = oracle.spmm_mean_f64(o[0], o[1], o[2], o[3], X)
    assert_mean_close(runs, ref, cond, what=f"task runs, K={K}, S={S}")
    assert_mean_close(warp, ref, cond, what=f"warp per task, K={K}, S={S}")
    tasks = torch.as_tensor(_DevTasks(p["t_ptr"], p["n_tasks"]), device="cuda:0").cpu().numpy()
    deg = np.diff(o[0])
    whole = []
    for rs, re_, fo, ln in tasks.reshape(-1, 4):
        for r in range(rs, re_):
            b = fo if r == rs else 0
            e = ln if (r == re_ - 1 and ln > 0) else deg[r]
            if b == 0 and e == deg[r]:
                whole.append(o[3][r])
    whole = np.array(whole, np.int64)
    assert len(whole) > n // 4
    assert np.array_equal(runs[whole].view(np.uint32), warp[whole].view(np.uint32))


def test_task_runs_keep_a_huge_hub_row_within_tolerance(ctx, oracle):
    """A row of degree 2^20 at S = 16 is cut into 65,536 fragment tasks.  Warp
    runs add each run's fragments in registers and reach the row with ~2,000
    float atomics instead of 65,536, which keeps the row within the
    condition-relative 1e-5 (one warp per task, forced, is reported beside it:
    its accumulated rounding is what the runs remove)."""
    rng = np.random.default_rng(41)
    hub = 1 << 20
    d = np.concatenate([rng.integers(0, 6, 20_000), [hub]])
    rowoff = np.zeros(len(d) + 1, np.int64)
    rowoff[1:] = np.cumsum(d)
    n_cols = hub
    col = rng.integers(0, n_cols, int(rowoff[-1])).astype(np.int32)
    col[rowoff[-2]:] = np.arange(hub, dtype=np.int32)  # the hub row: every column once
    rowoff = rowoff.astype(np.int32)
    val = np.ones(len(col), np.float32)
    K = 16
    # Positive features: the fragments' partial sums all share a sign, so the
    # float adds onto the hub's output row round in the same direction.
    X = graphs.uniform_features_np(n_cols, K, seed=42, lo=0.0, hi=1.0)
    costs = cs.SpmmCostParams(0.02, 0.7, 0.3, 0.5)
    p = _device_pipeline(ctx, rowoff, col, val, X, costs, 16)
    torch.cuda.synchronize()
    n, nnz = p["n"], p["nnz"]

    def run(flags):
        out = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda:0")
        ctx.spmm_mean_device(n, nnz, p["sro"].data_ptr(), p["scol"].data_ptr(), 0,
                             p["org"].data_ptr(), p["X"].data_ptr(), n_cols, K, p["t_ptr"],
                             p["n_tasks"], out.data_ptr(), cs.ROWS_COVERED | flags)
        torch.cuda.synchronize()
        assert ctx.take_device_errors() == 0
        return out.cpu().numpy()

    o = [t.cpu().numpy() for t in (p["sro"], p["scol"][:nnz], p["org"])]
    ref, cond = oracle.spmm_mean_f64(o[0], o[1], val, o[2], X)
    from helpers import rel_errors
    runs, warp = run(0), run(cs.TASK_PER_WARP)
    hub_row = len(d) - 1
    e_runs = float(rel_errors(runs[hub_row:hub_row + 1], ref[hub_row:hub_row + 1],
                              cond[hub_row:hub_row + 1]).max())
    e_warp = float(rel_errors(warp[hub_row:hub_row + 1], ref[hub_row:hub_row + 1],
                              cond[hub_row:hub_row + 1]).max())
    print(f"hub row of degree {hub}: warp runs {e_runs:.2e}, one warp per task {e_warp:.2e}")
    assert_mean_close(runs, ref, cond, what="warp runs, huge hub row")
    assert e_runs < e_warp
