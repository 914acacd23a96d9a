"""Direct CUDA forward operators for Gaussian CT splatting.

Public API identical to the reference (r2splat/ops/direct.py:10-69 for the
dataclasses, :120-135 ``prepare_inference_gaussians``, :222-251
``inference_rasterize``, :346-378 ``inference_voxelize``).

float32 inputs take the fused sm_100a path: one kernel for the parameter
transform + softplus, one for projection + conics/mu + tile rectangles
(which writes one 32-byte splat record per (view, Gaussian) instead of the
reference's means2d/cov2d/conics/mus/opacity tensors), the stable counting
binning, and the rasterizer.  float64 inputs run the reference's operator
chain (``r2splat.cuda._wrapper``) unchanged in order.  Both are GPU-only.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class InferenceGaussianState:
    """Reusable transformed Gaussian parameters for forward-only rendering."""

    covars: torch.Tensor
    max_scales: torch.Tensor
    opacities: torch.Tensor


@dataclass
class ProjectionRasterizationResult:
    image: torch.Tensor
    means2d: torch.Tensor
    radii: torch.Tensor


@dataclass
class MappingVoxelizationResult:
    volume: torch.Tensor
    means3d: torch.Tensor
    radii: torch.Tensor


@dataclass
class ProjectionForwardBuffers:
    """Forward state kept for the backward pass.

    float32: ``splats`` holds the per-(view, Gaussian) records
    (x, y, conic a, b, c, w*mu, cull extents); ``cov2d``, ``conics``,
    ``mus``, ``opacity`` and ``isect_ids`` are None.  float64: the
    reference's buffers are filled and ``splats`` is None.
    """

    output: torch.Tensor
    means2d: torch.Tensor
    radii: torch.Tensor
    tile_offsets: torch.Tensor
    flatten_ids: torch.Tensor
    viewmats: torch.Tensor
    Ks: torch.Tensor
    img_w: int
    img_h: int
    tile_size: int
    eps2d: float
    splats: Optional[torch.Tensor] = None
    # float32 with more intersection records than one int32 binning holds:
    # [(c0, c1, flatten_ids)] per contiguous view batch; the batch's rows of
    # tile_offsets index its own flatten_ids (flatten_ids above is then empty)
    view_batches: Optional[list] = None
    # float32 16x16 tiles, explicit (training) renders: the records' culling
    # ranges written by the forward for the backward (a tensor, or one per
    # view batch)
    cull: Optional[object] = None
    cov2d: Optional[torch.Tensor] = None
    conics: Optional[torch.Tensor] = None
    mus: Optional[torch.Tensor] = None
    opacity: Optional[torch.Tensor] = None
    isect_ids: Optional[torch.Tensor] = None


@dataclass
class VoxelForwardBuffers:
    """Voxel forward state (``vsplats`` for float32, reference buffers for float64)."""

    output: torch.Tensor
    means3d: torch.Tensor
    radii: torch.Tensor
    tile_offsets: torch.Tensor
    flatten_ids: torch.Tensor
    ranges: torch.Tensor
    centers: torch.Tensor
    dim2: int
    dim1: int
    dim0: int
    tile_size: int
    eps3d: float
    vsplats: Optional[torch.Tensor] = None
    conics: Optional[torch.Tensor] = None
    opacity: Optional[torch.Tensor] = None
    isect_ids: Optional[torch.Tensor] = None
    # float32 8-voxel bricks: per-record row table of the binning (r2s_voxel_rows_f32)
    rows: Optional[torch.Tensor] = None
    # brick layers [layer_begin, layer_end) along dim0 that were voxelized (a
    # z-slab; the whole grid by default): tile_offsets then holds those layers
    # only, indexing this slab's flatten_ids, and output their voxel rows
    layer_begin: int = 0
    layer_end: Optional[int] = None
    # float32: longest-first launch order of the bricks (r2s_brick_order)
    order: Optional[torch.Tensor] = None


def _fast(*tensors: torch.Tensor) -> bool:
    return all(t.dtype == torch.float32 for t in tensors)


@torch.no_grad()
def _prepare_forward_parameters(
    quats: torch.Tensor,
    raw_scales: torch.Tensor,
    raw_opacities: torch.Tensor,
    *,
    scale_min: float,
    scale_max: float,
) -> InferenceGaussianState:
    from ..cuda import _wrapper as W

    if not quats.is_cuda or not raw_scales.is_cuda or not raw_opacities.is_cuda:
        raise RuntimeError("Direct r2splat operators require CUDA tensors.")
    q = quats.contiguous()
    s = raw_scales.contiguous()
    o = raw_opacities.contiguous()
    if _fast(q, s, o) and q.dim() == 2 and q.size(1) == 4 and s.shape == (q.size(0), 3) \
            and o.shape == (q.size(0),):
        with torch.cuda.device(q.device):
            covars, max_scales, opacities = W.fused_prepare(q, s, o, scale_min, scale_max)
        return InferenceGaussianState(covars=covars, max_scales=max_scales, opacities=opacities)
    covars, max_scales = W.parameter_transform_fwd(q, s, float(scale_min), float(scale_max))
    opacities = torch.nn.functional.softplus(raw_opacities).contiguous()
    return InferenceGaussianState(covars=covars, max_scales=max_scales, opacities=opacities)


def prepare_inference_gaussians(
    quats: torch.Tensor,
    raw_scales: torch.Tensor,
    raw_opacities: torch.Tensor,
    *,
    scale_min: float,
    scale_max: float,
) -> InferenceGaussianState:
    """Transform raw parameters once for reusable forward-only evaluation."""
    return _prepare_forward_parameters(
        quats, raw_scales, raw_opacities, scale_min=scale_min, scale_max=scale_max
    )


def _tile_grid_2d(img_w: int, img_h: int, tile_size: int):
    if tile_size <= 0 or tile_size * tile_size > 1024:
        raise ValueError("2D tile_size must be positive with tile_size**2 <= 1024.")
    return (img_w + tile_size - 1) // tile_size, (img_h + tile_size - 1) // tile_size


@torch.no_grad()
def _rasterize_forward(
    means: torch.Tensor,
    covars: torch.Tensor,
    opacities: torch.Tensor,
    viewmats: torch.Tensor,
    Ks: torch.Tensor,
    *,
    img_w: int,
    img_h: int,
    tile_size: int,
    eps2d: float,
    radius_clip: float,
    keep_cull: bool = False,
) -> ProjectionForwardBuffers:
    from ..cuda import _wrapper as W

    img_w = int(img_w)
    img_h = int(img_h)
    tile_size = int(tile_size)
    ntx, nty = _tile_grid_2d(img_w, img_h, tile_size)
    means_c = means.contiguous()
    covars_c = covars.contiguous()
    viewmats_c = viewmats.contiguous()
    Ks_c = Ks.contiguous()
    n_cameras = int(viewmats_c.shape[0])
    if _fast(means_c, covars_c, opacities, viewmats_c, Ks_c):
        for name, t in (("means", means_c), ("covars", covars_c), ("opacities", opacities),
                        ("viewmats", viewmats_c), ("Ks", Ks_c)):
            if not t.is_cuda:
                raise RuntimeError(f"{name} must be a CUDA tensor")
        W._check_cameras(means_c, covars_c, viewmats_c, Ks_c)
        if float(radius_clip) <= 0.0:
            raise RuntimeError("radius_clip must be positive")
        N = means_c.size(0)
        opac = opacities.contiguous()
        if opac.shape != (N,):
            raise RuntimeError("opacities must be [N]")
        with torch.cuda.device(means_c.device):
            means2d, radii, splats, rects, _ = W.fused_project(
                means_c, covars_c, opac, viewmats_c, Ks_c, img_w, img_h, tile_size, ntx, nty,
                eps2d, radius_clip)
            T = ntx * nty
            limit = W.MAX_RECORDS_PER_BATCH if n_cameras > 1 else None
            binned = W.fused_bin(rects, n_cameras, N, T, ntx, 0, limit=limit)
            if binned is not None:
                offsets, flatten_ids, _ = binned
                tile_offsets = offsets.view(n_cameras, nty, ntx)
                cull = (torch.empty(flatten_ids.shape, dtype=torch.int16, device=means_c.device)
                        if keep_cull and tile_size == 16 else None)
                output = W.fused_raster_fwd(splats, tile_offsets, flatten_ids, n_cameras, N,
                                            img_w, img_h, tile_size, ntx, nty, cull=cull)
                view_batches = None
            else:
                # more records than one int32 binning holds: bin and rasterize
                # in contiguous view batches
                batches = W.plan_view_batches(rects, n_cameras, N, W.MAX_RECORDS_PER_BATCH)
                tile_offsets = torch.empty((n_cameras, nty, ntx), dtype=torch.int32,
                                           device=means_c.device)
                output = torch.empty((n_cameras, img_h, img_w), dtype=torch.float32,
                                     device=means_c.device)
                view_batches = []
                cull = [] if keep_cull and tile_size == 16 else None
                for c0, c1 in batches:
                    rb = rects[c0 * N * 8:c1 * N * 8]
                    binned = W.fused_bin(rb, c1 - c0, N, T, ntx, 0,
                                         limit=W.MAX_RECORDS_PER_BATCH)
                    if binned is None:
                        raise RuntimeError(
                            f"view {c0} alone holds more than {W.MAX_RECORDS_PER_BATCH} "
                            "intersection records (int32 tile offsets)")
                    offs_b, ids_b, _ = binned
                    tile_offsets[c0:c1] = offs_b.view(c1 - c0, nty, ntx)
                    cull_b = (torch.empty(ids_b.shape, dtype=torch.int16, device=means_c.device)
                              if cull is not None else None)
                    W.fused_raster_fwd(splats[c0:c1], tile_offsets[c0:c1], ids_b, c1 - c0, N,
                                       img_w, img_h, tile_size, ntx, nty, out=output[c0:c1],
                                       cull=cull_b)
                    view_batches.append((c0, c1, ids_b))
                    if cull is not None:
                        cull.append(cull_b)
                flatten_ids = torch.empty((0,), dtype=torch.int32, device=means_c.device)
        return ProjectionForwardBuffers(
            output=output, means2d=means2d, radii=radii, tile_offsets=tile_offsets,
            flatten_ids=flatten_ids, viewmats=viewmats_c, Ks=Ks_c, img_w=img_w, img_h=img_h,
            tile_size=tile_size, eps2d=float(eps2d), splats=splats, view_batches=view_batches,
            cull=cull)

    # reference operator chain (r2splat/ops/direct.py:166-201)
    means2d, cov2d, radii = W.world_to_image_projection_fwd(
        means_c, covars_c, viewmats_c, Ks_c, img_w, img_h, float(eps2d), float(radius_clip))
    conics, mus = W.conics_mu_fwd(cov2d, float(eps2d))
    opacity = opacities.unsqueeze(0).expand(n_cameras, -1).contiguous()
    _, isect_ids, flatten_ids = W.isect_tiles(means2d, radii, tile_size, ntx, nty)
    tile_offsets = W.isect_offset_encode(isect_ids, n_cameras, ntx, nty)
    output = W.rasterize_to_pixels_fwd(means2d, conics, opacity, mus, tile_offsets, flatten_ids,
                                       img_w, img_h, tile_size)
    return ProjectionForwardBuffers(
        output=output, means2d=means2d, radii=radii, tile_offsets=tile_offsets,
        flatten_ids=flatten_ids, viewmats=viewmats_c, Ks=Ks_c, img_w=img_w, img_h=img_h,
        tile_size=tile_size, eps2d=float(eps2d), cov2d=cov2d, conics=conics, mus=mus,
        opacity=opacity, isect_ids=isect_ids)


def inference_rasterize(
    state: InferenceGaussianState,
    means: torch.Tensor,
    viewmats: torch.Tensor,
    Ks: torch.Tensor,
    *,
    img_w: int,
    img_h: int,
    tile_size: int,
    eps2d: float,
    radius_clip: float,
) -> ProjectionRasterizationResult:
    """Rasterize without building or retaining any backward state."""
    buffers = _rasterize_forward(
        means, state.covars, state.opacities, viewmats, Ks, img_w=img_w, img_h=img_h,
        tile_size=tile_size, eps2d=eps2d, radius_clip=radius_clip)
    return ProjectionRasterizationResult(image=buffers.output, means2d=buffers.means2d,
                                         radii=buffers.radii)


def _tile_grid_3d(dim2: int, dim1: int, dim0: int, tile_size: int):
    if tile_size <= 0 or tile_size ** 3 > 1024:
        raise ValueError("3D tile_size must be positive with tile_size**3 <= 1024.")
    return ((dim2 + tile_size - 1) // tile_size, (dim1 + tile_size - 1) // tile_size,
            (dim0 + tile_size - 1) // tile_size)


@torch.no_grad()
def _voxelize_forward(
    means: torch.Tensor,
    covars: torch.Tensor,
    max_scales: torch.Tensor,
    opacities: torch.Tensor,
    ranges: torch.Tensor,
    centers: torch.Tensor,
    *,
    dim2: int,
    dim1: int,
    dim0: int,
    tile_size: int,
    eps3d: float,
    radius_clip: float,
    z_layers: Optional[tuple] = None,
) -> VoxelForwardBuffers:
    from ..cuda import _wrapper as W

    dim2, dim1, dim0, tile_size = int(dim2), int(dim1), int(dim0), int(tile_size)
    nt2, nt1, nt0 = _tile_grid_3d(dim2, dim1, dim0, tile_size)
    if z_layers is None:
        l0, l1 = 0, nt0
    else:
        l0, l1 = (int(v) for v in z_layers)
        if not 0 <= l0 <= l1 <= nt0:
            raise ValueError(f"z_layers must satisfy 0 <= begin <= end <= {nt0} brick layers.")
    means_c = means.contiguous()
    covars_c = covars.contiguous()
    ranges_c = ranges.contiguous()
    centers_c = centers.contiguous()
    if _fast(means_c, covars_c, opacities, ranges_c, centers_c):
        for name, t in (("means", means_c), ("covars", covars_c), ("opacities", opacities),
                        ("ranges", ranges_c), ("centers", centers_c)):
            if not t.is_cuda:
                raise RuntimeError(f"{name} must be a CUDA tensor")
        N = means_c.size(0)
        if means_c.dim() != 2 or means_c.size(1) != 3 or covars_c.shape != (N, 6):
            raise RuntimeError("means must be [N, 3] and covars [N, 6]")
        if ranges_c.shape != (3,) or centers_c.shape != (3,):
            raise RuntimeError("ranges and centers must be [3]")
        opac = opacities.contiguous()
        with torch.cuda.device(means_c.device):
            means3d, conics, radii, vsplats, rects, _ = W.fused_map(
                means_c, covars_c, opac, ranges_c, centers_c, dim2, dim1, dim0, tile_size, nt2,
                nt1, nt0, eps3d, radius_clip)
            # binning of layers [l0, l1) in the global key space (segment l0 first)
            offsets, flatten_ids, _ = W.fused_bin(rects, l1 - l0, N, nt1 * nt2, nt2, 1,
                                                  segment_base=l0)
            tile_offsets = offsets.view(l1 - l0, nt1, nt2)
            order = W.fused_brick_order(offsets, flatten_ids.numel())
            rows = W.fused_voxel_rows(vsplats, tile_offsets, flatten_ids, N, dim2, dim1, dim0,
                                      tile_size, nt2, nt1, nt0, l0, l1, order=order)
            output = W.fused_voxel_fwd(vsplats, tile_offsets, flatten_ids, N, dim2, dim1, dim0,
                                       tile_size, nt2, nt1, nt0, l0, l1, rows=rows, order=order)
        return VoxelForwardBuffers(
            output=output, means3d=means3d, radii=radii, tile_offsets=tile_offsets,
            flatten_ids=flatten_ids, ranges=ranges_c, centers=centers_c, dim2=dim2, dim1=dim1,
            dim0=dim0, tile_size=tile_size, eps3d=float(eps3d), vsplats=vsplats, conics=conics,
            opacity=opac, rows=rows, layer_begin=l0, layer_end=l1, order=order)

    if z_layers is not None and (l0, l1) != (0, nt0):
        raise RuntimeError("z_layers (a z-slab of the grid) needs float32 inputs")
    # reference operator chain (r2splat/ops/direct.py:284-326)
    means3d, conics, radii = W.world_to_volume_mapping_fwd(
        means_c, covars_c, max_scales.contiguous(), ranges_c, centers_c, dim2, dim1, dim0,
        float(eps3d), float(radius_clip))
    _, isect_ids, flatten_ids = W.isect_tiles_3d(means3d, radii, tile_size, nt2, nt1, nt0)
    tile_offsets = W.isect_offset_encode_3d(isect_ids, nt2, nt1, nt0)
    opacity = opacities.contiguous()
    output = W.voxelize_to_voxels_fwd(means3d, conics, opacity, tile_offsets, flatten_ids, dim2,
                                      dim1, dim0, tile_size)
    return VoxelForwardBuffers(
        output=output, means3d=means3d, radii=radii, tile_offsets=tile_offsets,
        flatten_ids=flatten_ids, ranges=ranges_c, centers=centers_c, dim2=dim2, dim1=dim1,
        dim0=dim0, tile_size=tile_size, eps3d=float(eps3d), conics=conics, opacity=opacity,
        isect_ids=isect_ids)


def inference_voxelize(
    state: InferenceGaussianState,
    means: torch.Tensor,
    ranges: torch.Tensor,
    centers: torch.Tensor,
    *,
    dim2: int,
    dim1: int,
    dim0: int,
    tile_size: int,
    eps3d: float,
    radius_clip: float,
) -> MappingVoxelizationResult:
    """Voxelize without building or retaining any backward state."""
    buffers = _voxelize_forward(
        means, state.covars, state.max_scales, state.opacities, ranges, centers, dim2=dim2,
        dim1=dim1, dim0=dim0, tile_size=tile_size, eps3d=eps3d, radius_clip=radius_clip)
    return MappingVoxelizationResult(volume=buffers.output, means3d=buffers.means3d,
                                     radii=buffers.radii)


__all__ = [
    "InferenceGaussianState",
    "MappingVoxelizationResult",
    "ProjectionRasterizationResult",
    "inference_rasterize",
    "inference_voxelize",
    "prepare_inference_gaussians",
]
