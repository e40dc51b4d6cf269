"""Row shards for running the aggregation on several GPUs of one node.

The path partitions without a data exchange: each rank takes a contiguous
block of ORIGINAL rows [a, b) whose summed full-row weight
(Cc + Cl) * deg + Cs -- the weight the reference's partitioner gives a whole
row (src/utils.cpp:850-852) -- is about 1/world of the total, sorts and
partitions that block on its own GPU, and aggregates it with the dense input
replicated.  Its output rows are a contiguous slice of the original-order
output, so no collective touches the data path.

When the dense input comes row-sharded from a prior layer (rank r holds rows
[a_r, b_r) of X: exactly the rows it produced), gather_rows rebuilds the full X
on every rank with one collective per call before the aggregation.
"""
from __future__ import annotations


def shard_bounds(rowoff, edge_weight: float, store_weight: float, world: int, rank: int):
    """[a, b) of rank `rank` out of `world`: the library's cost-balanced cut
    (cwlb_shard_bounds, the rule the multi-GPU entry points use) of the
    prefix sum of edge_weight * deg + store_weight at k/world of the total.
    Takes a torch tensor or a numpy array of row offsets (rows + 1)."""
    import numpy as np

    import cwlb_spmm as cs
    try:
        import torch
        if isinstance(rowoff, torch.Tensor):
            rowoff = rowoff.cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    n = len(rowoff) - 1
    if world <= 1:
        return 0, n
    costs = cs.SpmmCostParams(float(edge_weight), 0.0, float(store_weight), 0.0)
    b = cs.shard_bounds(np.asarray(rowoff), costs, world)
    return int(b[rank]), int(b[rank + 1])


def shard_csr(rowoff, col, val, a: int, b: int):
    """The sub-CSR of original rows [a, b): rebased offsets, column ids and
    values (columns still index the full, replicated dense input)."""
    e0, e1 = int(rowoff[a]), int(rowoff[b])
    ro = rowoff[a:b + 1] - e0
    return ro, col[e0:e1], val[e0:e1]


def gather_rows(x, bounds, group=None):
    """All-gather of a row-sharded matrix in place: on entry rank r holds rows
    bounds[r] = (a_r, b_r) of `x` (a contiguous [rows, K] tensor, the same
    shape on every rank); on return every rank holds all rows.  The blocks are
    uneven (cost-balanced shards), so the exchange is one broadcast per rank,
    issued together: NCCL runs them as one grouped call over NVLink; gloo (CPU
    tests) runs them in turn.  Returns x."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world <= 1:
        return x
    views = [x[a:b] for a, b in bounds]
    if dist.get_backend(group) == "nccl":
        rank = dist.get_rank(group)
        # Uneven output sizes: torch issues the per-rank broadcasts in one
        # NCCL group; the input is this rank's own block of x (no copy).
        dist.all_gather(views, views[rank], group=group)
    else:
        for r in range(world):
            if views[r].numel():
                dist.broadcast(views[r], src=r, group=group)
    return x
