"""Gaussian-only CT splatting operators (sm_100a build).

Drop-in for the reference package of the same name (r2splat/__init__.py):
the public names below and the submodules ``r2splat.ops``,
``r2splat.ops.direct``, ``r2splat.ops.explicit`` and
``r2splat.cuda._wrapper`` keep the reference's signatures.  All compute
runs in ``libr2s.so`` (hand-written sm_100a CUDA, C ABI in include/r2s.h).
"""

__version__ = "0.1.0"

from .ops import ExplicitGaussianState, InferenceGaussianState

__all__ = ["__version__", "ExplicitGaussianState", "InferenceGaussianState"]
