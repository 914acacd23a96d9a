"""Model-level adapter of the path: the four ``GaussianModel`` methods that
drive the operators (src/models/gaussian_model.py:280-492).

``GaussianAdapter`` holds the model's raw parameters (means [N,3], quats
[N,4], raw scales [N,3], raw opacities [N]) and operator settings and
restates, on the ``r2splat.ops`` of this package:

* ``prepare_gaussians(explicit=...)`` (:280-317): requires bounded sigmoid
  scales with scalar bounds (``RuntimeError`` otherwise) and returns the
  explicit (training) or inference state;
* ``rasterize(camtoworlds, Ks, width, height, ...)`` (:319-427): rejects
  ``packed``, ``sparse_grad``, a non-classic mode, a non-pinhole camera
  (``ValueError``) and extra options (``TypeError``); world-to-camera
  matrices are the rigid inverse of ``camtoworlds`` unless given (same shape
  required); returns renders [C, W, H, 1] (the [C, H, W] image with its last
  two axes swapped) and ``info`` = {means2d, radii.amax(-1), gaussian_ids
  [C, N] (an expanded cached arange), width, height, n_cameras};
* ``voxelize(volume_shape, bbox, ...)`` (:429-480): ``None`` without a bbox;
  ``volume_shape`` = (width, depth, height) -> dim2, dim1, dim0; ranges and
  centres from the [2, 3] bbox; returns the volume [dim0, dim1, dim2, 1];
* ``backward_explicit(state)`` (:482-492): ``TypeError`` for a non-explicit
  state, then the explicit backward into the four parameters' ``.grad``.

The parameters stay the caller's tensors (``torch.nn.Parameter`` in a
trainer), so optimisers, checkpoints (``r2s_checkpoint``) and strategies work
on them unchanged.
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple, Union

import torch

from r2splat.ops import (ExplicitGaussianState, InferenceGaussianState, inference_rasterize,
                         inference_voxelize)
from r2splat.ops.direct import prepare_inference_gaussians
from r2splat.ops.explicit import (explicit_backward, explicit_rasterize, explicit_voxelize,
                                  prepare_explicit_gaussians)


def invert_rigid_transform(transform: torch.Tensor) -> torch.Tensor:
    """[R^T | -R^T t] of [..., 4, 4] rigid transforms (src/utils/math.py:5-32);
    ``ValueError`` for another trailing shape."""
    if transform.shape[-2:] != (4, 4):
        raise ValueError(f"Expected transform shape [..., 4, 4], got {tuple(transform.shape)}")
    rt = transform[..., :3, :3].transpose(-1, -2)
    t = -(rt @ transform[..., :3, 3:4])
    out = torch.zeros(transform.shape, dtype=transform.dtype, device=transform.device)
    out[..., :3, :3] = rt
    out[..., :3, 3:4] = t
    out[..., 3, 3] = 1
    return out.contiguous()


class GaussianAdapter:
    """The operator-facing half of ``GaussianModel`` (see the module doc).

    Defaults are the reference's binary-tree model configuration: 16-pixel
    tiles, 8-voxel bricks, eps 1e-8 in 2D and 3D, radius clip 3, primitive
    backward, sigmoid scale bounds [5e-4, 1]."""

    def __init__(self, means: torch.Tensor, quats: torch.Tensor, scales: torch.Tensor,
                 opacities: torch.Tensor, *, scale_min: Optional[float] = 5e-4,
                 scale_max: Optional[float] = 1.0, img_tile_size: int = 16,
                 vol_tile_size: int = 8, eps2d: float = 1e-8, eps3d: float = 1e-8,
                 img_radius_clip: float = 3.0, vol_radius_clip: float = 3.0,
                 backward_mode: str = "primitive"):
        self.means, self.quats, self.scales, self.opacities = means, quats, scales, opacities
        self.scale_min, self.scale_max = scale_min, scale_max
        self.img_tile_size, self.vol_tile_size = img_tile_size, vol_tile_size
        self.eps2d, self.eps3d = eps2d, eps3d
        self.img_radius_clip, self.vol_radius_clip = img_radius_clip, vol_radius_clip
        self.backward_mode = backward_mode
        self._gaussian_ids_cache: Optional[torch.Tensor] = None

    @property
    def device(self) -> torch.device:
        return self.means.device

    @property
    def num_gaussians(self) -> int:
        return int(self.means.shape[0])

    def prepare_gaussians(self, *, explicit: bool = False
                          ) -> Union[InferenceGaussianState, ExplicitGaussianState]:
        if self.scale_min is None or self.scale_max is None:
            raise RuntimeError("Direct r2splat operators require bounded sigmoid scales.")
        smin = torch.as_tensor(self.scale_min)
        smax = torch.as_tensor(self.scale_max)
        if smin.numel() != 1 or smax.numel() != 1:
            raise RuntimeError("Direct r2splat operators require scalar scale bounds.")
        smin, smax = float(smin.item()), float(smax.item())
        if explicit:
            return prepare_explicit_gaussians(self.quats, self.scales, self.opacities,
                                              scale_min=smin, scale_max=smax,
                                              backward_mode=self.backward_mode)
        return prepare_inference_gaussians(self.quats, self.scales, self.opacities,
                                           scale_min=smin, scale_max=smax)

    def rasterize(self, camtoworlds: torch.Tensor, Ks: torch.Tensor, width: int, height: int,
                  packed: bool = False, sparse_grad: bool = False, absgrad: bool = False,
                  rasterize_mode: str = "classic", camera_model: str = "pinhole",
                  viewmats: Optional[torch.Tensor] = None,
                  gaussian_state: Optional[Union[InferenceGaussianState,
                                                 ExplicitGaussianState]] = None,
                  **kwargs) -> Tuple[torch.Tensor, Dict[str, Any]]:
        if packed:
            raise ValueError("r2splat does not support packed=True.")
        if sparse_grad:
            raise ValueError("r2splat does not support sparse_grad=True.")
        if rasterize_mode != "classic":
            raise ValueError("r2splat only supports rasterize_mode='classic'.")
        if camera_model != "pinhole":
            raise ValueError("r2splat only supports camera_model='pinhole'.")
        if kwargs:
            raise TypeError(f"Unsupported rasterization options: {sorted(kwargs)}")
        if viewmats is None:
            viewmats = invert_rigid_transform(camtoworlds)
        if viewmats.shape != camtoworlds.shape:
            raise ValueError("viewmats must have the same shape as camtoworlds, got "
                             f"{tuple(viewmats.shape)} and {tuple(camtoworlds.shape)}.")
        state = gaussian_state if gaussian_state is not None else self.prepare_gaussians()
        args = dict(img_w=width, img_h=height, tile_size=self.img_tile_size, eps2d=self.eps2d,
                    radius_clip=self.img_radius_clip)
        if isinstance(state, ExplicitGaussianState):
            result = explicit_rasterize(state, self.means, viewmats, Ks, absgrad=absgrad, **args)
        elif isinstance(state, InferenceGaussianState):
            result = inference_rasterize(state, self.means, viewmats, Ks, **args)
        else:
            raise TypeError("gaussian_state must be an InferenceGaussianState or "
                            "ExplicitGaussianState.")
        n_cameras = int(camtoworlds.shape[0])
        info = {
            "means2d": result.means2d,
            "radii": result.radii.amax(dim=-1),
            "gaussian_ids": self._gaussian_ids(n_cameras),
            "width": int(width),
            "height": int(height),
            "n_cameras": n_cameras,
        }
        return result.image.transpose(1, 2).unsqueeze(-1).contiguous(), info

    def voxelize(self, volume_shape: Tuple[int, int, int], bbox: Optional[torch.Tensor],
                 gaussian_state: Optional[Union[InferenceGaussianState,
                                                ExplicitGaussianState]] = None,
                 **kwargs) -> Optional[torch.Tensor]:
        if bbox is None:
            return None
        if kwargs:
            raise TypeError(f"Unsupported voxelization options: {sorted(kwargs)}")
        width, depth, height = volume_shape
        box = bbox.to(self.device)
        ranges = box[1] - box[0]
        centers = (box[0] + box[1]) / 2.0
        state = gaussian_state if gaussian_state is not None else self.prepare_gaussians()
        args = dict(dim2=width, dim1=depth, dim0=height, tile_size=self.vol_tile_size,
                    eps3d=self.eps3d, radius_clip=self.vol_radius_clip)
        if isinstance(state, ExplicitGaussianState):
            result = explicit_voxelize(state, self.means, ranges, centers, **args)
        elif isinstance(state, InferenceGaussianState):
            result = inference_voxelize(state, self.means, ranges, centers, **args)
        else:
            raise TypeError("gaussian_state must be an InferenceGaussianState or "
                            "ExplicitGaussianState.")
        return result.volume.unsqueeze(-1).contiguous()

    def backward_explicit(self, gaussian_state: ExplicitGaussianState, **kwargs) -> None:
        """Explicit backward into the four parameters; keyword options (e.g.
        ``densify=``) pass through to ``explicit_backward``."""
        if not isinstance(gaussian_state, ExplicitGaussianState):
            raise TypeError("backward_explicit requires an ExplicitGaussianState.")
        explicit_backward(gaussian_state, self.means, self.quats, self.scales, self.opacities,
                          **kwargs)

    def _gaussian_ids(self, n_cameras: int) -> torch.Tensor:
        cache = self._gaussian_ids_cache
        if cache is None or cache.device != self.means.device or cache.numel() != self.num_gaussians:
            cache = torch.arange(self.num_gaussians, device=self.means.device, dtype=torch.long)
            self._gaussian_ids_cache = cache
        return cache.expand(n_cameras, -1)
