"""Seeded synthetic CSR graphs and feature matrices for the CWLB-SpMM configs.

The reference evaluates on 19 external `.csr` graphs that are not part of its
repository; these generators stand in for them with the shapes, sizes and
degree distributions that the benchmark configurations name:

  er        Erdos-Renyi G(n, p), directed, no self-loops (config 1)
  rmat      R-MAT(a, b, c, d) edge sampling over 2^scale vertices, optionally
            self-loop-free, symmetrised and de-duplicated (configs 2 and 5)
  poisson   per-row degree ~ Poisson(mean), uniform columns (config 3)
  geometric per-row degree ~ Geometric(1/mean) clipped to max_degree,
            uniform columns (config 4)

Every generator returns (row_offset int32[N+1], col_ind int32[nnz],
value float32[nnz]) with unit values and ascending column ids in each row,
the layout of the reference's CSR (include/Matrix.h:15-26, values set to 1.0
by src/data.cpp:115).

Two back ends produce the same distributions: numpy (CPU; small cases,
tests) and torch (CUDA or CPU; the multi-GB bench configs).  They use
different random streams, so the same seed gives different graphs on the two
back ends; every consumer builds its input once and feeds that one copy to
both the device path and the checker.
"""
from __future__ import annotations

import numpy as np


# ---------------------------------------------------------------------------
# numpy back end

def _csr_from_edges_np(n_rows, src, dst):
    order = np.lexsort((dst, src))
    src, dst = src[order], dst[order]
    counts = np.bincount(src, minlength=n_rows)
    rowoff = np.zeros(n_rows + 1, np.int64)
    np.cumsum(counts, out=rowoff[1:])
    if rowoff[-1] >= 2**31:
        raise OverflowError("nnz does not fit the reference's int32 CSR")
    return (rowoff.astype(np.int32), dst.astype(np.int32),
            np.ones(len(dst), np.float32))


def er_np(n, avg_degree, seed):
    """Directed Erdos-Renyi with p = avg_degree / (n - 1), no self-loops."""
    rng = np.random.default_rng(seed)
    p = avg_degree / max(n - 1, 1)
    src_l, dst_l = [], []
    block = max(1, (1 << 24) // max(n, 1))
    for r0 in range(0, n, block):
        r1 = min(n, r0 + block)
        m = rng.random((r1 - r0, n)) < p
        rr, cc = np.nonzero(m)
        rr = rr + r0
        keep = rr != cc
        src_l.append(rr[keep])
        dst_l.append(cc[keep])
    return _csr_from_edges_np(n, np.concatenate(src_l), np.concatenate(dst_l))


def rmat_np(scale, n_edges, a, b, c, seed, symmetrize=False, drop_self_loops=False,
            dedupe=False):
    """R-MAT edge sampling (quadrant probabilities a, b, c, 1-a-b-c)."""
    rng = np.random.default_rng(seed)
    n = 1 << scale
    src = np.zeros(n_edges, np.int64)
    dst = np.zeros(n_edges, np.int64)
    for level in range(scale):
        r = rng.random(n_edges)
        bit = 1 << (scale - 1 - level)
        down = r >= a + b                      # quadrants c, d
        right = ((r >= a) & (r < a + b)) | (r >= a + b + c)  # quadrants b, d
        src += down * bit
        dst += right * bit
    if drop_self_loops:
        keep = src != dst
        src, dst = src[keep], dst[keep]
    if symmetrize:
        src, dst = np.concatenate([src, dst]), np.concatenate([dst, src])
    if dedupe:
        key = np.unique(src * n + dst)
        src, dst = key // n, key % n
    return _csr_from_edges_np(n, src, dst)


def degree_graph_np(degrees, n_cols, seed):
    """Rows with the given degrees and uniform random columns (sorted)."""
    rng = np.random.default_rng(seed)
    degrees = np.asarray(degrees, np.int64)
    n = len(degrees)
    rowoff = np.zeros(n + 1, np.int64)
    np.cumsum(degrees, out=rowoff[1:])
    col = rng.integers(0, n_cols, rowoff[-1])
    src = np.repeat(np.arange(n), degrees)
    order = np.lexsort((col, src))
    return rowoff.astype(np.int32), col[order].astype(np.int32), np.ones(rowoff[-1], np.float32)


def poisson_np(n, mean, seed):
    rng = np.random.default_rng(seed)
    return degree_graph_np(rng.poisson(mean, n), n, seed + 1)


def geometric_np(n, mean, max_degree, seed):
    rng = np.random.default_rng(seed)
    d = np.minimum(rng.geometric(1.0 / mean, n), max_degree)
    return degree_graph_np(d, n, seed + 1)


def uniform_features_np(rows, cols, seed, lo=-1.0, hi=1.0):
    return np.random.default_rng(seed).uniform(lo, hi, (rows, cols)).astype(np.float32)


def normal_features_np(rows, cols, seed):
    return np.random.default_rng(seed).standard_normal((rows, cols), dtype=np.float32)


# ---------------------------------------------------------------------------
# torch back end (large configs; runs on the GPU when device="cuda")

def _csr_from_edges_torch(torch, n_rows, src, dst, device):
    key = src * n_rows + dst
    key, _ = torch.sort(key)
    src = key // n_rows
    dst = key - src * n_rows
    counts = torch.bincount(src, minlength=n_rows)
    rowoff = torch.zeros(n_rows + 1, dtype=torch.int64, device=device)
    torch.cumsum(counts, 0, out=rowoff[1:])
    if int(rowoff[-1]) >= 2**31:
        raise OverflowError("nnz does not fit the reference's int32 CSR")
    return rowoff.to(torch.int32), dst.to(torch.int32), torch.ones(
        dst.numel(), dtype=torch.float32, device=device)


def rmat_torch(scale, n_edges, a, b, c, seed, device="cuda", symmetrize=False,
               drop_self_loops=False, dedupe=False, chunk=1 << 26):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    n = 1 << scale
    srcs, dsts = [], []
    for e0 in range(0, n_edges, chunk):
        m = min(chunk, n_edges - e0)
        src = torch.zeros(m, dtype=torch.int64, device=device)
        dst = torch.zeros(m, dtype=torch.int64, device=device)
        for level in range(scale):
            r = torch.rand(m, generator=g, device=device)
            bit = 1 << (scale - 1 - level)
            down = r >= a + b
            right = ((r >= a) & (r < a + b)) | (r >= a + b + c)
            src += down.to(torch.int64) * bit
            dst += right.to(torch.int64) * bit
        srcs.append(src)
        dsts.append(dst)
    src = torch.cat(srcs)
    dst = torch.cat(dsts)
    del srcs, dsts
    if drop_self_loops:
        keep = src != dst
        src, dst = src[keep], dst[keep]
    if symmetrize:
        src, dst = torch.cat([src, dst]), torch.cat([dst, src])
    if dedupe:
        key = torch.unique(src * n + dst)
        src, dst = key // n, key % n
    return _csr_from_edges_torch(torch, n, src, dst, device)


def degree_graph_torch(degrees, n_cols, seed, device="cuda"):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    degrees = degrees.to(device=device, dtype=torch.int64)
    n = degrees.numel()
    rowoff = torch.zeros(n + 1, dtype=torch.int64, device=device)
    torch.cumsum(degrees, 0, out=rowoff[1:])
    nnz = int(rowoff[-1])
    if nnz >= 2**31:
        raise OverflowError("nnz does not fit the reference's int32 CSR")
    col = torch.randint(0, n_cols, (nnz,), generator=g, device=device, dtype=torch.int64)
    src = torch.repeat_interleave(torch.arange(n, device=device), degrees)
    key, _ = torch.sort(src * n_cols + col)
    col = (key - src * n_cols).to(torch.int32)
    return rowoff.to(torch.int32), col, torch.ones(nnz, dtype=torch.float32, device=device)


def poisson_torch(n, mean, seed, device="cuda"):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    rates = torch.full((n,), float(mean), device=device)
    deg = torch.poisson(rates, generator=g).to(torch.int64)
    return degree_graph_torch(deg, n, seed + 1, device)


def geometric_torch(n, mean, max_degree, seed, device="cuda"):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    u = torch.rand(n, generator=g, device=device, dtype=torch.float64).clamp_min(1e-300)
    p = 1.0 / mean
    deg = (torch.floor(torch.log(u) / np.log1p(-p)) + 1).clamp(1, max_degree).to(torch.int64)
    return degree_graph_torch(deg, n, seed + 1, device)


def uniform_features_torch(rows, cols, seed, device="cuda", lo=-1.0, hi=1.0):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.empty((rows, cols), dtype=torch.float32, device=device)
    x.uniform_(lo, hi, generator=g)
    return x


def normal_features_torch(rows, cols, seed, device="cuda"):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.empty((rows, cols), dtype=torch.float32, device=device)
    x.normal_(0.0, 1.0, generator=g)
    return x


# ---------------------------------------------------------------------------
# the benchmark configurations
#
# S: the segment size both bench arms (the GPU path and the CPU reference
# arm) partition with, so that they time the same task list.  Configurations
# 2-5 use the third candidate of the reference's --candidates procedure
# (wave_based_s with the nnz-keyed w table, main.cpp:87-95 and 295-321, at
# w = 2048 and 148 SMs), the candidate that procedure keeps on a B200 (for
# configuration 2, S = 181 times within 1% of it).

CONFIGS = {
    1: dict(name="er4096_k32", graph=("er", dict(n=4096, avg_degree=8, seed=0)),
            K=32, features=("uniform", 0), S=32),
    # R-MAT directed samples before self-loop removal, symmetrisation and
    # de-duplication; 6.2e7 samples leave ~1.1e8 stored nonzeros.
    2: dict(name="rmat18_k128", graph=("rmat", dict(scale=18, n_edges=85_000_000, a=0.57,
                                                     b=0.19, c=0.19, seed=1, symmetrize=True,
                                                     drop_self_loops=True, dedupe=True)),
            K=128, features=("uniform", 1), S=362),
    3: dict(name="poisson2.4m_k512", graph=("poisson", dict(n=2_400_000, mean=51, seed=2)),
            K=512, features=("normal", 2), S=404),
    4: dict(name="geom16m_k32", graph=("geometric", dict(n=1 << 24, mean=4, max_degree=200,
                                                          seed=3)),
            K=32, features=("uniform", 3), S=222),
    5: dict(name="rmat22_k64", graph=("rmat", dict(scale=22, n_edges=1 << 28, a=0.70, b=0.10,
                                                    c=0.10, seed=4)),
            K=64, features=("uniform", 4), S=886),
}


def build_config_torch(cfg_id, device="cuda", scale_down=1):
    """CSR (+ features) of a benchmark configuration, built with torch.

    scale_down > 1 shrinks the vertex and edge counts by that factor (used for
    profiling captures that must stay small); 1 builds the configuration as
    specified.
    """
    cfg = CONFIGS[cfg_id]
    kind, p = cfg["graph"]
    p = dict(p)
    if kind == "er":
        rowoff, col, val = (np.asarray(x) for x in er_np(**p))
        import torch
        rowoff, col, val = (torch.from_numpy(x).to(device) for x in (rowoff, col, val))
        n = p["n"]
    elif kind == "rmat":
        if scale_down > 1:
            shift = int(np.log2(scale_down))
            p["scale"] -= shift
            p["n_edges"] //= scale_down
        rowoff, col, val = rmat_torch(device=device, **p)
        n = 1 << p["scale"]
    elif kind == "poisson":
        p["n"] //= scale_down
        rowoff, col, val = poisson_torch(device=device, **p)
        n = p["n"]
    else:
        p["n"] //= scale_down
        rowoff, col, val = geometric_torch(device=device, **p)
        n = p["n"]
    fk, fseed = cfg["features"]
    if fk == "uniform":
        X = uniform_features_torch(n, cfg["K"], fseed, device)
    else:
        X = normal_features_torch(n, cfg["K"], fseed, device)
    return rowoff, col, val, X
