"""Explicit first-order Gaussian CT splatting.

Same contract as the reference (r2splat/ops/explicit.py:1-394): the CUDA
forward pass is detached from autograd, the rendered image and volume are
leaf tensors that any PyTorch loss can differentiate, and
:func:`explicit_backward` applies the Gaussian VJP once and accumulates
gradients into the raw parameters (means, quats, raw scales, raw
opacities), setting ``means2d.grad`` (and ``.absgrad``) for densification.

float32 backward is two kernels: the rasterizer / voxelizer statistics and
one fused per-Gaussian kernel that performs the reference's chain
conics_mu_bwd -> world_to_image_projection_bwd -> (sum over views) ->
world_to_volume_mapping_bwd -> parameter_transform_bwd -> softplus VJP
(explicit.py:277-384) and accumulates into ``.grad`` in place.  float64
runs the reference's operator chain.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .direct import (
    MappingVoxelizationResult,
    ProjectionForwardBuffers,
    ProjectionRasterizationResult,
    VoxelForwardBuffers,
    _prepare_forward_parameters,
    _rasterize_forward,
    _voxelize_forward,
)


def _validate_backward_mode(backward_mode: str) -> str:
    mode = str(backward_mode).lower()
    if mode not in {"pixel", "primitive"}:
        raise ValueError("backward_mode must be 'pixel' or 'primitive'.")
    return mode


@dataclass
class ExplicitProjectionContext:
    output: torch.Tensor
    means2d: torch.Tensor
    buffers: ProjectionForwardBuffers
    absgrad: bool


@dataclass
class ExplicitVoxelContext:
    output: torch.Tensor
    buffers: VoxelForwardBuffers


@dataclass
class ExplicitGaussianState:
    """One-shot context shared by projection and voxelization for one step."""

    covars: torch.Tensor
    max_scales: torch.Tensor
    opacities: torch.Tensor
    scale_min: float
    scale_max: float
    backward_mode: str
    projection: Optional[ExplicitProjectionContext] = None
    voxel: Optional[ExplicitVoxelContext] = None
    backward_called: bool = False


def prepare_explicit_gaussians(
    quats: torch.Tensor,
    raw_scales: torch.Tensor,
    raw_opacities: torch.Tensor,
    *,
    scale_min: float,
    scale_max: float,
    backward_mode: str = "primitive",
) -> ExplicitGaussianState:
    """Activate raw parameters without constructing a renderer autograd graph."""
    mode = _validate_backward_mode(backward_mode)
    prepared = _prepare_forward_parameters(
        quats, raw_scales, raw_opacities, scale_min=scale_min, scale_max=scale_max)
    return ExplicitGaussianState(
        covars=prepared.covars,
        max_scales=prepared.max_scales,
        opacities=prepared.opacities,
        scale_min=float(scale_min),
        scale_max=float(scale_max),
        backward_mode=mode,
    )


def explicit_rasterize(
    state: ExplicitGaussianState,
    means: torch.Tensor,
    viewmats: torch.Tensor,
    Ks: torch.Tensor,
    *,
    img_w: int,
    img_h: int,
    tile_size: int,
    eps2d: float,
    radius_clip: float,
    absgrad: bool,
) -> ProjectionRasterizationResult:
    """Run the Gaussian projection/rasterization forward path explicitly."""
    if state.projection is not None:
        raise RuntimeError("An explicit Gaussian state can only be rasterized once.")
    buffers = _rasterize_forward(
        means, state.covars, state.opacities, viewmats, Ks, img_w=img_w, img_h=img_h,
        tile_size=tile_size, eps2d=eps2d, radius_clip=radius_clip, keep_cull=True)
    output = buffers.output.detach().requires_grad_(True)
    means2d = buffers.means2d.detach().requires_grad_(True)
    state.projection = ExplicitProjectionContext(
        output=output, means2d=means2d, buffers=buffers, absgrad=bool(absgrad))
    return ProjectionRasterizationResult(image=output, means2d=means2d, radii=buffers.radii)


def explicit_voxelize(
    state: ExplicitGaussianState,
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
    z_layers: Optional[tuple] = None,
) -> MappingVoxelizationResult:
    """Run the Gaussian mapping/voxelization forward path explicitly.

    ``z_layers`` is an extension of this build (the reference has no such
    argument; leaving it out gives the reference's behaviour): a brick-layer
    range ``(begin, end)`` along dim0 voxelizes only that z-slab of the grid,
    in the grid's own key space -- one rank's share of a multi-GPU split.
    The volume is then the slab's voxel rows ``[min(end*tile, dim0) -
    begin*tile, dim1, dim2]`` and the backward takes that slab's gradient.
    float32 only."""
    if state.voxel is not None:
        raise RuntimeError("An explicit Gaussian state can only be voxelized once.")
    buffers = _voxelize_forward(
        means, state.covars, state.max_scales, state.opacities, ranges, centers, dim2=dim2,
        dim1=dim1, dim0=dim0, tile_size=tile_size, eps3d=eps3d, radius_clip=radius_clip,
        z_layers=z_layers)
    output = buffers.output.detach().requires_grad_(True)
    state.voxel = ExplicitVoxelContext(output=output, buffers=buffers)
    return MappingVoxelizationResult(volume=output, means3d=buffers.means3d, radii=buffers.radii)


def _accumulate_grad(parameter: torch.Tensor, grad: torch.Tensor) -> None:
    grad = grad.detach()
    if parameter.grad is None:
        parameter.grad = grad
    else:
        parameter.grad.add_(grad)


def _inplace_grad_ok(parameter: torch.Tensor) -> bool:
    """True when the existing .grad can be accumulated into by the fused kernel."""
    g = parameter.grad
    return (g is not None and g.dtype == torch.float32 and g.is_contiguous()
            and g.shape == parameter.shape and g.device == parameter.device)


@torch.no_grad()
def explicit_backward(
    state: ExplicitGaussianState,
    means: torch.Tensor,
    quats: torch.Tensor,
    raw_scales: torch.Tensor,
    raw_opacities: torch.Tensor,
    *,
    densify=None,
) -> None:
    """Apply the saved first-order CUDA VJP and accumulate raw parameter grads.

    ``densify`` (an ``r2splat.ops.training.DensifyAccumulator``, float32
    renders only) additionally accumulates the densification statistics of
    the render in the same kernel; without it the behaviour is the
    reference's (r2splat/ops/explicit.py:233-385)."""
    if state.backward_called:
        raise RuntimeError("Explicit first-order backward can only run once per state.")
    if state.projection is None:
        raise RuntimeError("Explicit backward requires a projection forward pass.")
    proj = state.projection
    pb = proj.buffers
    if pb.splats is not None:
        _explicit_backward_fused(state, means, quats, raw_scales, raw_opacities, densify)
    else:
        if densify is not None:
            raise RuntimeError("explicit_backward: fused densification statistics need a "
                               "float32 render")
        _explicit_backward_chain(state, means, quats, raw_scales, raw_opacities)
    state.backward_called = True


def _explicit_backward_fused(state, means, quats, raw_scales, raw_opacities,
                             densify=None) -> None:
    from ..cuda import _wrapper as W

    proj = state.projection
    pb = proj.buffers
    C, N = pb.means2d.size(0), pb.means2d.size(1)
    dev = pb.means2d.device
    ntx, nty = pb.tile_offsets.size(2), pb.tile_offsets.size(1)
    with torch.cuda.device(dev):
        v_image = proj.output.grad
        raster_stats = None
        if v_image is not None:
            v_image = v_image.contiguous()
            if pb.view_batches is None:
                raster_stats = W.fused_raster_bwd(
                    pb.splats, pb.tile_offsets, pb.flatten_ids, v_image, C, N, pb.img_w,
                    pb.img_h, pb.tile_size, ntx, nty, proj.absgrad, cull=pb.cull)
            else:
                raster_stats = torch.empty((C * N, 8), dtype=torch.float32, device=dev)
                for k, (c0, c1, ids_b) in enumerate(pb.view_batches):
                    W.fused_raster_bwd(pb.splats[c0:c1], pb.tile_offsets[c0:c1], ids_b,
                                       v_image[c0:c1], c1 - c0, N, pb.img_w, pb.img_h,
                                       pb.tile_size, ntx, nty, proj.absgrad,
                                       out=raster_stats[c0 * N:c1 * N],
                                       cull=pb.cull[k] if pb.cull is not None else None)
            v_means2d = torch.empty((C, N, 2), dtype=torch.float32, device=dev)
            v_means2d_abs = (torch.empty((C, N, 2), dtype=torch.float32, device=dev)
                             if proj.absgrad else None)
        else:
            v_means2d = torch.zeros_like(proj.means2d)
            v_means2d_abs = torch.zeros_like(proj.means2d) if proj.absgrad else None
        store = densify is None or densify.store_screen_grads
        if densify is not None and densify.absgrad and not proj.absgrad:
            raise RuntimeError("explicit_backward: densify with absgrad needs a render with "
                               "absgrad=True")
        if not store:
            v_means2d = v_means2d_abs = None
        dens_args = (None if densify is None
                     else densify.launch_args(pb.radii.contiguous(), pb.img_w, pb.img_h))

        vox = state.voxel
        vox_stats = None
        vb = None
        if vox is not None and vox.output.grad is not None:
            vb = vox.buffers
            nt0 = (vb.dim0 + vb.tile_size - 1) // vb.tile_size
            vox_stats = W.fused_voxel_bwd(
                vb.vsplats, vb.tile_offsets, vb.flatten_ids, vox.output.grad.contiguous(), N,
                vb.dim2, vb.dim1, vb.dim0, vb.tile_size, vb.tile_offsets.size(2),
                vb.tile_offsets.size(1), nt0, vb.layer_begin,
                nt0 if vb.layer_end is None else vb.layer_end, rows=vb.rows, order=vb.order)

        params = (means, quats, raw_scales, raw_opacities)
        accumulate = all(_inplace_grad_ok(p) for p in params)
        if accumulate:
            outs = [p.grad for p in params]
        else:
            outs = [torch.empty(p.shape, dtype=torch.float32, device=dev) for p in params]
        W.fused_explicit_backward(
            means.contiguous(), quats.contiguous(), raw_scales.contiguous(),
            raw_opacities.contiguous(), state.scale_min, state.scale_max, pb.viewmats, pb.Ks,
            pb.img_w, pb.img_h, pb.eps2d, raster_stats, v_means2d if raster_stats is not None else None,
            v_means2d_abs if raster_stats is not None else None,
            vb.ranges if vb is not None else None, vb.centers if vb is not None else None,
            vb.dim2 if vb is not None else 0, vb.dim1 if vb is not None else 0,
            vb.dim0 if vb is not None else 0, vb.eps3d if vb is not None else 0.0, vox_stats,
            accumulate, outs, densify=dens_args)
    if store:
        proj.means2d.grad = v_means2d.detach()
        if proj.absgrad:
            proj.means2d.absgrad = v_means2d_abs.detach()
    if not accumulate:
        for p, g in zip((means, quats, raw_scales, raw_opacities), outs):
            _accumulate_grad(p, g)


def _explicit_backward_chain(state, means, quats, raw_scales, raw_opacities) -> None:
    """Reference operator chain (r2splat/ops/explicit.py:258-384)."""
    from ..cuda import _wrapper as W

    v_means_total = torch.zeros_like(means)
    v_covars_total = torch.zeros_like(state.covars)
    v_opacity_total = torch.zeros_like(state.opacities)
    proj = state.projection
    pb = proj.buffers
    v_image = proj.output.grad
    if v_image is None:
        v_means2d = torch.zeros_like(proj.means2d)
        v_means2d_abs = torch.zeros_like(proj.means2d) if proj.absgrad else None
    else:
        args = (pb.means2d, pb.conics, pb.opacity, pb.mus, pb.tile_offsets)
        if state.backward_mode == "primitive":
            grads = W.rasterize_to_pixels_bwd_per_gaussian(
                *args, pb.isect_ids, pb.flatten_ids, v_image.contiguous(), pb.img_w, pb.img_h,
                pb.tile_size, proj.absgrad)
        else:
            grads = W.rasterize_to_pixels_bwd(
                *args, pb.flatten_ids, v_image.contiguous(), pb.img_w, pb.img_h, pb.tile_size,
                proj.absgrad)
        v_means2d_abs, v_means2d, v_conics, v_opacity, v_mus = grads
        v_cov2d = W.conics_mu_bwd(pb.cov2d, pb.eps2d, pb.conics, pb.mus, v_conics.contiguous(),
                                  v_mus.contiguous())
        v_means, v_covars = W.world_to_image_projection_bwd(
            means.contiguous(), state.covars, pb.viewmats, pb.Ks, pb.img_w, pb.img_h,
            v_means2d.contiguous(), v_cov2d.contiguous())
        v_means_total.add_(v_means)
        v_covars_total.add_(v_covars)
        v_opacity_total.add_(v_opacity.sum(dim=0))
    proj.means2d.grad = v_means2d.detach()
    if proj.absgrad:
        proj.means2d.absgrad = v_means2d_abs.detach()

    vox = state.voxel
    if vox is not None and vox.output.grad is not None:
        vb = vox.buffers
        args = (vb.means3d, vb.conics, vb.opacity, vb.tile_offsets)
        if state.backward_mode == "primitive":
            v_m3, v_c3, v_o3 = W.voxelize_to_voxels_bwd_per_gaussian(
                *args, vb.isect_ids, vb.flatten_ids, vox.output.grad.contiguous(), vb.dim2,
                vb.dim1, vb.dim0, vb.tile_size)
        else:
            v_m3, v_c3, v_o3 = W.voxelize_to_voxels_bwd(
                *args, vb.flatten_ids, vox.output.grad.contiguous(), vb.dim2, vb.dim1, vb.dim0,
                vb.tile_size)
        v_means, v_covars = W.world_to_volume_mapping_bwd(
            means.contiguous(), state.covars, vb.ranges, vb.centers, vb.dim2, vb.dim1, vb.dim0,
            vb.eps3d, v_m3.contiguous(), v_c3.contiguous())
        v_means_total.add_(v_means)
        v_covars_total.add_(v_covars)
        v_opacity_total.add_(v_o3)

    v_quats, v_raw_scales = W.parameter_transform_bwd(
        quats.contiguous(), raw_scales.contiguous(), state.scale_min, state.scale_max,
        v_covars_total.contiguous())
    v_raw_opacities = v_opacity_total * torch.sigmoid(raw_opacities)
    _accumulate_grad(means, v_means_total)
    _accumulate_grad(quats, v_quats)
    _accumulate_grad(raw_scales, v_raw_scales)
    _accumulate_grad(raw_opacities, v_raw_opacities)


__all__ = [
    "ExplicitGaussianState",
    "explicit_backward",
    "explicit_rasterize",
    "explicit_voxelize",
    "prepare_explicit_gaussians",
]
