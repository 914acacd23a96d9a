"""Drive the live reference build (oracle/_ref) -- TEST INFRASTRUCTURE ONLY.

``oracle/build_ref.py`` compiles the reference's own CUDA sources for sm_100a
into ``oracle/_ref/r2splat_ref_csrc.so`` (a pybind11 module exposing the 18
reference operators, r2splat/cuda/csrc/ext.cpp:7-27).  This module loads it
and calls those operators in the order of the reference's op layer:

* ``prepare``           -- r2splat/ops/direct.py:93-117
* ``rasterize_forward`` -- r2splat/ops/direct.py:138-219
* ``voxelize_forward``  -- r2splat/ops/direct.py:254-343
* ``explicit_backward`` -- r2splat/ops/explicit.py:233-385

It is used by the GPU parity tests (bit-exact integer outputs, float
tolerances) and by ``bench.py --impl reference``.  The product package never
imports it.
"""

from __future__ import annotations

import importlib.util
import os
from typing import Optional

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "r2splat_ref_csrc.so")


def reference_available(path: str = REF_SO) -> bool:
    return os.path.exists(path)


def load_reference_module(path: str = REF_SO):
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"reference build not found at {path}; run `python oracle/build_ref.py` where the "
            "reference sources are available")
    spec = importlib.util.spec_from_file_location("r2splat_ref_csrc", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class ReferencePipeline:
    """The reference op layer's call sequence on the reference's own kernels."""

    def __init__(self, module=None):
        self.C = module if module is not None else load_reference_module()

    # direct.py:93-117
    @torch.no_grad()
    def prepare(self, quats, raw_scales, raw_opacities, scale_min, scale_max):
        covars, max_scales = self.C.parameter_transform_fwd(
            quats.contiguous(), raw_scales.contiguous(), float(scale_min), float(scale_max))
        opac = torch.nn.functional.softplus(raw_opacities).contiguous()
        return covars, max_scales, opac

    # direct.py:138-219
    @torch.no_grad()
    def rasterize_forward(self, means, covars, opacities, viewmats, Ks, img_w, img_h, tile_size,
                          eps2d, radius_clip):
        C = self.C
        means2d, cov2d, radii = C.world_to_image_projection_fwd(
            means.contiguous(), covars.contiguous(), viewmats.contiguous(), Ks.contiguous(),
            img_w, img_h, float(eps2d), float(radius_clip))
        conics, mus = C.conics_mu_fwd(cov2d, float(eps2d))
        n_cameras = int(viewmats.shape[0])
        opacity = opacities.unsqueeze(0).expand(n_cameras, -1).contiguous()
        nty = (img_h + tile_size - 1) // tile_size
        ntx = (img_w + tile_size - 1) // tile_size
        tiles_per_gauss, isect_ids, flatten_ids = C.isect_tiles(means2d, radii, tile_size, ntx, nty)
        tile_offsets = C.isect_offset_encode(isect_ids, n_cameras, ntx, nty)
        output = C.rasterize_to_pixels_fwd(means2d, conics, opacity, mus, tile_offsets,
                                           flatten_ids, img_w, img_h, tile_size)
        return dict(output=output, means2d=means2d, cov2d=cov2d, conics=conics, mus=mus,
                    opacity=opacity, radii=radii, tiles_per_gauss=tiles_per_gauss,
                    tile_offsets=tile_offsets, flatten_ids=flatten_ids, isect_ids=isect_ids,
                    viewmats=viewmats.contiguous(), Ks=Ks.contiguous(), img_w=img_w, img_h=img_h,
                    tile_size=tile_size, eps2d=float(eps2d))

    # direct.py:254-343
    @torch.no_grad()
    def voxelize_forward(self, means, covars, max_scales, opacities, ranges, centers, dim2, dim1,
                         dim0, tile_size, eps3d, radius_clip):
        C = self.C
        means3d, conics, radii = C.world_to_volume_mapping_fwd(
            means.contiguous(), covars.contiguous(), max_scales.contiguous(), ranges.contiguous(),
            centers.contiguous(), dim2, dim1, dim0, float(eps3d), float(radius_clip))
        nt2 = (dim2 + tile_size - 1) // tile_size
        nt1 = (dim1 + tile_size - 1) // tile_size
        nt0 = (dim0 + tile_size - 1) // tile_size
        tiles_per_gauss, isect_ids, flatten_ids = C.isect_tiles_3d(means3d, radii, tile_size, nt2,
                                                                   nt1, nt0)
        tile_offsets = C.isect_offset_encode_3d(isect_ids, nt2, nt1, nt0)
        opacity = opacities.contiguous()
        output = C.voxelize_to_voxels_fwd(means3d, conics, opacity, tile_offsets, flatten_ids,
                                          dim2, dim1, dim0, tile_size)
        return dict(output=output, means3d=means3d, conics=conics, opacity=opacity, radii=radii,
                    tiles_per_gauss=tiles_per_gauss, tile_offsets=tile_offsets,
                    flatten_ids=flatten_ids, isect_ids=isect_ids, ranges=ranges.contiguous(),
                    centers=centers.contiguous(), dim2=dim2, dim1=dim1, dim0=dim0,
                    tile_size=tile_size, eps3d=float(eps3d))

    # explicit.py:233-385 ("primitive" or "pixel" backward mode)
    @torch.no_grad()
    def explicit_backward(self, proj: Optional[dict], v_image, vox: Optional[dict], v_volume,
                          means, quats, raw_scales, raw_opacities, covars, opacities, scale_min,
                          scale_max, absgrad=False, mode="primitive"):
        C = self.C
        v_means_total = torch.zeros_like(means)
        v_covars_total = torch.zeros_like(covars)
        v_opacity_total = torch.zeros_like(opacities)
        v_means2d = v_means2d_abs = None
        if proj is not None and v_image is not None:
            args = (proj["means2d"], proj["conics"], proj["opacity"], proj["mus"],
                    proj["tile_offsets"])
            if mode == "primitive":
                grads = C.rasterize_to_pixels_bwd_per_gaussian(
                    *args, proj["isect_ids"], proj["flatten_ids"], v_image.contiguous(),
                    proj["img_w"], proj["img_h"], proj["tile_size"], absgrad)
            else:
                grads = C.rasterize_to_pixels_bwd(
                    *args, proj["flatten_ids"], v_image.contiguous(), proj["img_w"],
                    proj["img_h"], proj["tile_size"], absgrad)
            v_means2d_abs, v_means2d, v_conics, v_opacity, v_mus = grads
            v_cov2d = C.conics_mu_bwd(proj["cov2d"], proj["eps2d"], proj["conics"], proj["mus"],
                                      v_conics.contiguous(), v_mus.contiguous())
            v_means, v_covars = C.world_to_image_projection_bwd(
                means.contiguous(), covars, proj["viewmats"], proj["Ks"], proj["img_w"],
                proj["img_h"], v_means2d.contiguous(), v_cov2d.contiguous())
            v_means_total.add_(v_means)
            v_covars_total.add_(v_covars)
            v_opacity_total.add_(v_opacity.sum(dim=0))
        if vox is not None and v_volume is not None:
            args = (vox["means3d"], vox["conics"], vox["opacity"], vox["tile_offsets"])
            if mode == "primitive":
                v_m3, v_c3, v_o3 = C.voxelize_to_voxels_bwd_per_gaussian(
                    *args, vox["isect_ids"], vox["flatten_ids"], v_volume.contiguous(),
                    vox["dim2"], vox["dim1"], vox["dim0"], vox["tile_size"])
            else:
                v_m3, v_c3, v_o3 = C.voxelize_to_voxels_bwd(
                    *args, vox["flatten_ids"], v_volume.contiguous(), vox["dim2"], vox["dim1"],
                    vox["dim0"], vox["tile_size"])
            v_means, v_covars = C.world_to_volume_mapping_bwd(
                means.contiguous(), covars, vox["ranges"], vox["centers"], vox["dim2"],
                vox["dim1"], vox["dim0"], vox["eps3d"], v_m3.contiguous(), v_c3.contiguous())
            v_means_total.add_(v_means)
            v_covars_total.add_(v_covars)
            v_opacity_total.add_(v_o3)
        v_quats, v_raw_scales = C.parameter_transform_bwd(
            quats.contiguous(), raw_scales.contiguous(), float(scale_min), float(scale_max),
            v_covars_total.contiguous())
        v_raw_opac = v_opacity_total * torch.sigmoid(raw_opacities)
        return dict(means=v_means_total, quats=v_quats, scales=v_raw_scales, opacities=v_raw_opac,
                    means2d=v_means2d, means2d_abs=v_means2d_abs)
