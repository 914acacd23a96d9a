"""Host-side sharding of the r2splat hot path over one process per GPU.

Projection: the views of one orbit are dealt to the ranks, every world-th view
starting at the rank's index (``view_split``: the job's views split across
the GPUs, strong scaling; ``view_shard``: every rank renders the same number
of views of a world-times-larger orbit, weak scaling), so that each rank's
views span the whole circle and see the same amount of the scene (contiguous
arcs differ by several per cent in intersection records); the raw-parameter
gradients are summed across ranks;
the gradient is linear in the per-view contributions, so the sum equals the
single-process gradient over all views.  Voxelization: the brick layers of
the grid are split into contiguous z-slabs, one per rank; a rank bins only its
layers (in the global key space) and voxelizes its slab.  The gradient sum is
the only collective of the path.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch


def view_shard(views_per_rank: int, rank: int, world: int) -> Tuple[int, int, int, int]:
    """(first view, view count, orbit size, stride) of `rank`'s views: views
    first, first + stride, ... of the orbit."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return rank, views_per_rank, views_per_rank * world, world


def view_split(n_views: int, rank: int, world: int) -> Tuple[int, int, int, int]:
    """(first view, view count, orbit size, stride) of `rank`'s share of a job
    of `n_views` views: views rank, rank + world, ... of that orbit (ranks
    hold ceil or floor of n_views / world views)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return rank, len(range(rank, n_views, world)), n_views, world


def layer_range(n_layers: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous brick-layer range [l0, l1) of `rank`; ranks beyond the
    layers get an empty range."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    per = (n_layers + world - 1) // world
    l0 = min(n_layers, rank * per)
    return l0, min(n_layers, l0 + per)


def balanced_layer_ranges(weights: Sequence[float], world: int) -> List[Tuple[int, int]]:
    """Contiguous brick-layer ranges, one per rank, minimizing the largest
    total weight (records per layer) of any rank: binary search on that
    maximum with greedy packing as the feasibility test.  Deterministic: every
    rank computes the same ranges from the same weights."""
    n = len(weights)
    if world < 1:
        raise ValueError("world must be positive")
    w = [max(0.0, float(x)) for x in weights]
    total = sum(w)
    if total <= 0.0:
        return [layer_range(n, r, world) for r in range(world)]

    def pack(cap):
        ranges, start, acc = [], 0, 0.0
        for i, x in enumerate(w):
            if acc + x > cap and i > start:
                ranges.append((start, i))
                start, acc = i, 0.0
            acc += x
        ranges.append((start, n))
        return ranges

    lo, hi = max(w), total
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if len(pack(mid)) <= world:
            hi = mid
        else:
            lo = mid
    ranges = pack(hi)
    ranges += [(n, n)] * (world - len(ranges))
    return ranges


def layer_weights(rects3: torch.Tensor, n_layers: int) -> List[float]:
    """Records per brick layer from the packed 3D brick rectangles
    ([N] x 16 bytes: x0|x1<<16, y0|y1<<16, z0|z1<<16, pad, as the volume
    mapping writes them): each Gaussian adds its x-y brick area to every layer
    of its z range."""
    r = rects3.view(torch.int32).view(-1, 4)[:, :3].to(torch.int64) & 0xFFFFFFFF
    lo, hi = r & 0xFFFF, r >> 16
    area = ((hi[:, 0] - lo[:, 0]).clamp_min(0) * (hi[:, 1] - lo[:, 1]).clamp_min(0)).double()
    z0 = lo[:, 2].clamp(0, n_layers)
    z1 = hi[:, 2].clamp(0, n_layers)
    ok = z1 > z0
    diff = torch.zeros(n_layers + 1, dtype=torch.float64, device=rects3.device)
    diff.scatter_add_(0, z0[ok], area[ok])
    diff.scatter_add_(0, z1[ok], -area[ok])
    return torch.cumsum(diff, 0)[:n_layers].tolist()


# Time of a brick layer beyond its records, in records: its 3D binning, row
# table and brick launches cost about as much per brick as 94 records do in
# the voxel forward and backward (a fit of t = a + b records + c layers to the
# eight z-slabs of config 2 on 8 B200s: b = 0.31 ms per million records,
# c = 0.030 ms per layer of 1,024 bricks).
BRICK_COST_RECORDS = 94.0


def layer_costs(rects3: torch.Tensor, n_layers: int, bricks_per_layer: int) -> List[float]:
    """Weights of the z-slab split: records per brick layer plus the layer's
    own cost (BRICK_COST_RECORDS per brick), so that ranks of many sparse
    layers are not given as many records as ranks of a few dense ones."""
    extra = BRICK_COST_RECORDS * bricks_per_layer
    return [x + extra for x in layer_weights(rects3, n_layers)]


def slab_rows(l0: int, l1: int, tile: int, dim0: int) -> Tuple[int, int]:
    """Voxel rows [z0, z1) of brick layers [l0, l1) in a grid of depth dim0."""
    z0 = l0 * tile
    return z0, max(z0, min(l1 * tile, dim0))


class GradientAllReduce:
    """Sums a list of gradient tensors across ranks with one all-reduce of a
    reused flat buffer (same collective on every rank, same order)."""

    def __init__(self, group=None):
        self.group = group
        self.flat = None

    def __call__(self, grads: Sequence[torch.Tensor]) -> List[torch.Tensor]:
        import torch.distributed as dist

        n = sum(g.numel() for g in grads)
        if (self.flat is None or self.flat.numel() != n or self.flat.device != grads[0].device
                or self.flat.dtype != grads[0].dtype):
            self.flat = torch.empty(n, device=grads[0].device, dtype=grads[0].dtype)
        off = 0
        for g in grads:
            self.flat[off:off + g.numel()].copy_(g.reshape(-1))
            off += g.numel()
        dist.all_reduce(self.flat, group=self.group)
        off = 0
        for g in grads:
            g.copy_(self.flat[off:off + g.numel()].view_as(g))
            off += g.numel()
        return list(grads)


def data_parallel_objective(out: dict, w_l1: float, w_ssim: float, w_tv: float,
                            n_local_views: int, n_total_views: int, world: int,
                            w_hierarchy: float = 0.0) -> torch.Tensor:
    """The scalar a rank backpropagates so that the sum of the ranks'
    gradients equals the one-process gradient of the training loss
    (BinaryTreeLossComputer, src/utils/loss.py:125-172, including its
    ``w_hierarchy * hierarchy`` term) over all the step's views.  ``out`` is
    the loss computer's dict for this rank's views.

    L1, SSIM and the edge term are means over (view, pixel) with per-view
    SSIM windows, so a rank's mean over its own views weighted by
    n_local / n_total sums to the mean over all views.  Every rank evaluates
    the same TV sub-volume, so TV is weighted 1 / world; the hierarchy loss
    (src/utils/loss.py:27-60) depends only on the replicated parameters and
    the archived parents, so it is weighted 1 / world as well."""
    frac = float(n_local_views) / float(n_total_views)
    proj = w_l1 * out["proj_l1"] + w_ssim * out["proj_ssim"] + out["edge_weight"] * out["edge"]
    total = frac * proj + (w_tv / float(world)) * out["vol_tv"]
    if w_hierarchy and "hierarchy" in out:
        total = total + (float(w_hierarchy) / float(world)) * out["hierarchy"]
    return total
