"""Lazy ctypes loader of ``libr2s.so``.

Same contract as the reference loader (r2splat/cuda/_backend.py:9-58):
importing never touches CUDA; the first attribute access loads the library
only when ``torch.cuda.is_available()``; when it cannot be used every access
raises ``RuntimeError``.  There is no CPU fallback.

The library path can be overridden with the ``R2S_LIBRARY`` environment
variable; by default it is ``r2splat/_lib/libr2s.so`` next to this package
(built by ``bt-3dgs_b200/build.py``).
"""

from __future__ import annotations

import ctypes
import os

import torch

_LIB_PATH = os.environ.get(
    "R2S_LIBRARY",
    os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib", "libr2s.so"),
)

_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_f64 = ctypes.c_double
_p = ctypes.c_void_p

class AdamGroup(ctypes.Structure):
    """r2s_adam_group of include/r2s.h."""

    _fields_ = [("param", ctypes.c_void_p), ("grad", ctypes.c_void_p),
                ("exp_avg", ctypes.c_void_p), ("exp_avg_sq", ctypes.c_void_p),
                ("numel", ctypes.c_int64), ("lr", ctypes.c_double), ("step", ctypes.c_int64)]


class DensifyArgs(ctypes.Structure):
    """r2s_densify_args of include/r2s.h."""

    _fields_ = [("radii", ctypes.c_void_p), ("scale_x", ctypes.c_double),
                ("scale_y", ctypes.c_double), ("extent", ctypes.c_double),
                ("absgrad", ctypes.c_int32), ("grad2d", ctypes.c_void_p),
                ("count", ctypes.c_void_p), ("max_radii", ctypes.c_void_p)]


# argument type lists of every exported function (include/r2s.h)
_SIGNATURES = {
    "r2s_version": ([], ctypes.c_char_p),
    "r2s_adam_step_f32": ([ctypes.POINTER(AdamGroup), _i32, _f64, _f64, _f64, _p], _i32),
    "r2s_densify_stats_f32": ([_p, _p, _i64, _i64, _f64, _f64, _f64, _p, _p, _p, _p], _i32),
    "r2s_projection_loss_f32": (
        [_p, _p, _p, _p, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _p], _i32),
    "r2s_tv_loss_f32": ([_p, _i64, _i64, _i64, _p, _p, _p, _p], _i32),
    "r2s_projection_loss_combine_f32": ([_p, _p, _p, _p, _p, _i64, _p, _p, _p], _i32),
    "r2s_last_error": ([ctypes.c_char_p, ctypes.c_size_t], ctypes.c_size_t),
    "r2s_split_children_f32": (
        [_p, _p, _p, _p, _p, _i64, _f64, _f64, _f64, _i32, _p, _p, _p, _p, _p], _i32),
    "r2s_debug_build": ([], _i32),
    "r2s_debug_flags": ([ctypes.POINTER(ctypes.c_uint32), _i32], _i32),
    "r2s_calib_ffma_f32": ([_p, _i64, _i32, _p], _i32),
    "r2s_calib_ex2_f32": ([_p, _i64, _i32, _p], _i32),
    "r2s_parameter_transform_fwd": ([_i32, _p, _p, _f64, _f64, _p, _p, _i64, _p], _i32),
    "r2s_parameter_transform_bwd": ([_i32, _p, _p, _f64, _f64, _p, _p, _p, _i64, _p], _i32),
    "r2s_world_to_image_projection_fwd": (
        [_i32, _p, _p, _p, _p, _i64, _i64, _u32, _u32, _f64, _f64, _p, _p, _p, _p], _i32),
    "r2s_world_to_image_projection_bwd": (
        [_i32, _p, _p, _p, _p, _i64, _i64, _u32, _u32, _p, _p, _p, _p, _p], _i32),
    "r2s_conics_mu_fwd": ([_i32, _p, _f64, _p, _p, _i64, _p], _i32),
    "r2s_conics_mu_bwd": ([_i32, _p, _f64, _p, _p, _p, _p, _p, _i64, _p], _i32),
    "r2s_world_to_volume_mapping_fwd": (
        [_i32, _p, _p, _p, _p, _p, _i64, _u32, _u32, _u32, _f64, _f64, _p, _p, _p, _p], _i32),
    "r2s_world_to_volume_mapping_bwd": (
        [_i32, _p, _p, _p, _p, _i64, _u32, _u32, _u32, _f64, _p, _p, _p, _p, _p], _i32),
    "r2s_bin_workspace_bytes": ([_i64, _i64, _i64, _i32], _i64),
    "r2s_isect_tiles_prepare": (
        [_i32, _p, _p, _i32, _i64, _i64, _u32, _u32, _u32, _p, _p, _p, _i64, _p, _p, _p], _i32),
    "r2s_isect_tiles_3d_prepare": (
        [_i32, _p, _p, _i64, _u32, _u32, _u32, _u32, _p, _p, _p, _i64, _p, _p, _p], _i32),
    "r2s_bin_prepare": ([_p, _i64, _i64, _i64, _u32, _i32, _i64, _p, _i64, _p, _p, _p], _i32),
    "r2s_bin_place": (
        [_p, _i64, _i64, _i64, _u32, _i32, _i64, _p, _i64, _p, _i64, _p, _p, _p], _i32),
    "r2s_isect_offset_encode": ([_p, _i64, _i64, _p, _p], _i32),
    "r2s_rasterize_to_pixels_fwd": (
        [_i32, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _p, _p, _p],
        _i32),
    "r2s_rasterize_to_pixels_bwd": (
        [_i32, _i32, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _u32, _u32, _u32, _u32, _u32,
         _p, _p, _p, _p, _p, _p, _p, _p], _i32),
    "r2s_rasterize_to_pixels_bwd_noalloc_f32": (
        [_i32, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _p, _p,
         _p, _p, _p, _p], _i32),
    "r2s_voxelize_to_voxels_fwd": (
        [_i32, _p, _p, _p, _p, _p, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _p, _p],
        _i32),
    "r2s_voxelize_to_voxels_bwd": (
        [_i32, _i32, _p, _p, _p, _p, _p, _p, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _u32,
         _p, _p, _p, _p, _p], _i32),
    "r2s_prepare_gaussians_f32": ([_p, _p, _p, _f64, _f64, _p, _p, _p, _i64, _p], _i32),
    "r2s_project_splats_f32": (
        [_p, _p, _p, _p, _p, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _f64, _f64, _p, _p, _p, _p,
         _p, _p], _i32),
    "r2s_raster_splats_fwd_f32": (
        [_p, _p, _p, _i64, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _p, _p, _p], _i32),
    "r2s_raster_splats_bwd_f32": (
        [_p, _p, _p, _p, _i64, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _i32, _p, _p, _p], _i32),
    "r2s_map_vsplats_f32": (
        [_p, _p, _p, _p, _p, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _f64, _f64, _p, _p,
         _p, _p, _p, _p, _p], _i32),
    "r2s_voxel_rows_f32": (
        [_p, _p, _p, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _p, _p,
         _p], _i32),
    "r2s_brick_order": ([_p, _i64, _i64, _p, _p], _i32),
    "r2s_voxel_splats_fwd_f32": (
        [_p, _p, _p, _p, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _p,
         _p, _p], _i32),
    "r2s_voxel_splats_bwd_f32": (
        [_p, _p, _p, _p, _p, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _u32,
         _p, _p, _p], _i32),
    "r2s_explicit_backward_f32": (
        [_p, _p, _p, _p, _f64, _f64, _p, _p, _i64, _i64, _u32, _u32, _f64, _p, _p, _p, _p, _p,
         _u32, _u32, _u32, _f64, _p, _i32, _p, _p, _p, _p, _p], _i32),
    "r2s_explicit_backward_densify_f32": (
        [_p, _p, _p, _p, _f64, _f64, _p, _p, _i64, _i64, _u32, _u32, _f64, _p, _p, _p, _p, _p,
         _u32, _u32, _u32, _f64, _p, _i32, _p, _p, _p, _p, ctypes.POINTER(DensifyArgs), _p],
        _i32),
}

UNAVAILABLE_MESSAGE = (
    "r2splat CUDA extension is unavailable. Build the sm_100a library with "
    "`python bt-3dgs_b200/build.py` and run on a machine with a CUDA GPU."
)


def load_library(path: str = _LIB_PATH) -> ctypes.CDLL:
    """Load ``libr2s.so`` and declare its C signatures (no CUDA call)."""
    lib = ctypes.CDLL(path)
    for name, (argtypes, restype) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


class _LazyLibrary:
    def __init__(self) -> None:
        self._lib = None
        self._load_attempted = False
        self._error = None

    def _try_load(self) -> None:
        if self._load_attempted:
            return
        self._load_attempted = True
        if not torch.cuda.is_available():
            return
        try:
            self._lib = load_library()
        except OSError as exc:  # missing or unloadable library
            self._lib = None
            self._error = str(exc)

    def __getattr__(self, name: str):
        self._try_load()
        if self._lib is None:
            detail = f" ({self._error})" if self._error else ""
            raise RuntimeError(UNAVAILABLE_MESSAGE + detail)
        return getattr(self._lib, name)

    def is_available(self) -> bool:
        self._try_load()
        return self._lib is not None


_lazy_C = _LazyLibrary()


class _CProxy:
    def __getattr__(self, name: str):
        return getattr(_lazy_C, name)

    def __bool__(self) -> bool:
        return _lazy_C.is_available()


_C = _CProxy()


def is_cuda_available() -> bool:
    return _lazy_C.is_available()


def library_path() -> str:
    return _LIB_PATH


__all__ = ["_C", "is_cuda_available", "load_library", "library_path", "UNAVAILABLE_MESSAGE"]
