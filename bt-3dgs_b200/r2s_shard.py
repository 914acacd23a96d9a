"""Host-side sharding of the r2splat hot path over one process per GPU.

Projection: every rank renders its own contiguous block of views of a shared
orbit (weak scaling) and the raw-parameter gradients are summed across ranks;
the gradient is linear in the per-view contributions, so the sum equals the
single-process gradient over all views.  Voxelization: the brick layers of
the grid are split into contiguous z-slabs, one per rank; a rank bins only its
layers (in the global key space) and voxelizes its slab.  The gradient sum is
the only collective of the path.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch


def view_shard(views_per_rank: int, rank: int, world: int) -> Tuple[int, int, int]:
    """(first view, view count, orbit size) of `rank`'s block of views."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return rank * views_per_rank, views_per_rank, views_per_rank * world


def layer_range(n_layers: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous brick-layer range [l0, l1) of `rank`; ranks beyond the
    layers get an empty range."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    per = (n_layers + world - 1) // world
    l0 = min(n_layers, rank * per)
    return l0, min(n_layers, l0 + per)


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
