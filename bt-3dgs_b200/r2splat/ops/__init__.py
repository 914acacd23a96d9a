"""Direct Gaussian CT splatting interfaces (reference: r2splat/ops/__init__.py)."""

from .direct import (
    InferenceGaussianState,
    MappingVoxelizationResult,
    ProjectionRasterizationResult,
    inference_rasterize,
    inference_voxelize,
    prepare_inference_gaussians,
)
from .explicit import ExplicitGaussianState

__all__ = [
    "ExplicitGaussianState",
    "InferenceGaussianState",
    "MappingVoxelizationResult",
    "ProjectionRasterizationResult",
    "inference_rasterize",
    "inference_voxelize",
    "prepare_inference_gaussians",
]
