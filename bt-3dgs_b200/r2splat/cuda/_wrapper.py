"""The reference's 18 low-level operators on top of ``libr2s.so``.

Each function keeps the positional signature, return order, dtypes and shapes
of the reference binding of the same name (r2splat/cuda/csrc/ext.cpp:7-27,
r2splat/cuda/include/Ops.h:9-79) and raises ``RuntimeError`` where the
reference's ``TORCH_CHECK`` would.  Outputs are allocated with torch on the
inputs' device; the kernels run on ``torch.cuda.current_stream()``.

Besides the 18 operators this module holds the fused float32 helpers used by
``r2splat.ops`` (prefixed ``fused_``); they are not part of the reference API.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

from ._backend import _C, is_cuda_available

_F32 = 0
_F64 = 1
_RECT2_BYTES = 8
_RECT3_BYTES = 16


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def _check_cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _dtype_code(t: torch.Tensor, op: str) -> int:
    if t.dtype == torch.float32:
        return _F32
    if t.dtype == torch.float64:
        return _F64
    raise RuntimeError(f'"{op}" not implemented for \'{t.dtype}\'')


def _same_dtype(op: str, ref: torch.Tensor, *others: torch.Tensor) -> None:
    for o in others:
        if o.dtype != ref.dtype:
            raise RuntimeError(f"{op}: expected all floating inputs to be {ref.dtype}, got {o.dtype}")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    _C.r2s_last_error(buf, 2048)
    return buf.value.decode(errors="replace")


# One NVTX range per library call, named after the C entry point, when the
# environment sets R2S_NVTX to anything but "0" (read once, at import): every
# stage of the path then shows up on profiler timelines.  Off by default.
_NVTX = os.environ.get("R2S_NVTX", "0") not in ("", "0")


def _call(fn_name: str, *args) -> None:
    if _NVTX:
        torch.cuda.nvtx.range_push(fn_name)
        try:
            rc = getattr(_C, fn_name)(*args)
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        rc = getattr(_C, fn_name)(*args)
    if rc != 0:
        raise RuntimeError(_last_error() or f"{fn_name} failed with status {rc}")


def _u32(v, name: str) -> int:
    v = int(v)
    if v < 0 or v > 0xFFFFFFFF:
        raise TypeError(f"{name} must be a non-negative 32-bit integer, got {v}")
    return v


def _bin_workspace(device, S: int, N: int, T: int, layered: int) -> torch.Tensor:
    nbytes = int(_C.r2s_bin_workspace_bytes(S, N, T, layered))
    _require(nbytes >= 0, "binning: invalid sizes")
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


def _read_count(n_dev: torch.Tensor) -> int:
    """One host read of the device-side intersection count (the reference
    syncs at the same point, csrc/IsectTiles.cpp:100)."""
    return int(n_dev.item())


# ---------------------------------------------------------------------------
# parameter transform
# ---------------------------------------------------------------------------
def parameter_transform_fwd(quats, scale_ori, scale_min, scale_max):
    _check_cuda("quats", quats)
    _check_cuda("scale_ori", scale_ori)
    _require(quats.dim() == 2 and quats.size(1) == 4,
             f"quats must be 2D [N, 4], got shape {list(quats.shape)}")
    _require(scale_ori.dim() == 2 and scale_ori.size(1) == 3,
             f"scale_ori must be 2D [N, 3], got shape {list(scale_ori.shape)}")
    N = quats.size(0)
    _require(scale_ori.size(0) == N,
             f"scale_ori batch dim ({scale_ori.size(0)}) doesn't match quats N={N}")
    code = _dtype_code(quats, "parameter_transform_fwd")
    _same_dtype("parameter_transform_fwd", quats, scale_ori)
    covars = torch.empty((N, 6), dtype=quats.dtype, device=quats.device)
    max_scales = torch.empty((N,), dtype=quats.dtype, device=quats.device)
    if N:
        with torch.cuda.device(quats.device):
            _call("r2s_parameter_transform_fwd", code, _ptr(quats), _ptr(scale_ori),
                  float(scale_min), float(scale_max), _ptr(covars), _ptr(max_scales), N,
                  _stream(quats.device))
    return covars, max_scales


def parameter_transform_bwd(quats, scale_ori, scale_min, scale_max, v_covars):
    _check_cuda("quats", quats)
    _check_cuda("scale_ori", scale_ori)
    _check_cuda("v_covars", v_covars)
    _require(quats.dim() == 2 and quats.size(1) == 4, "quats must be 2D [N, 4]")
    _require(scale_ori.dim() == 2 and scale_ori.size(1) == 3, "scale_ori must be 2D [N, 3]")
    _require(v_covars.dim() == 2 and v_covars.size(1) == 6, "v_covars must be 2D [N, 6]")
    N = quats.size(0)
    _require(scale_ori.size(0) == N and v_covars.size(0) == N, "Batch dimension mismatch")
    code = _dtype_code(quats, "parameter_transform_bwd")
    _same_dtype("parameter_transform_bwd", quats, scale_ori, v_covars)
    v_quats = torch.empty((N, 4), dtype=quats.dtype, device=quats.device)
    v_scale = torch.empty((N, 3), dtype=quats.dtype, device=quats.device)
    if N:
        with torch.cuda.device(quats.device):
            _call("r2s_parameter_transform_bwd", code, _ptr(quats), _ptr(scale_ori),
                  float(scale_min), float(scale_max), _ptr(v_covars), _ptr(v_quats),
                  _ptr(v_scale), N, _stream(quats.device))
    return v_quats, v_scale


# ---------------------------------------------------------------------------
# projection and conics
# ---------------------------------------------------------------------------
def _check_cameras(means, covars, viewmats, Ks):
    _require(means.dim() == 2 and means.size(1) == 3, "means must be [N, 3]")
    _require(covars.dim() == 2 and covars.size(1) == 6, "covars must be [N, 6]")
    _require(viewmats.dim() == 3 and viewmats.size(1) == 4 and viewmats.size(2) == 4,
             "viewmats must be [C, 4, 4]")
    _require(Ks.dim() == 3 and Ks.size(1) == 3 and Ks.size(2) == 3, "Ks must be [C, 3, 3]")
    _require(covars.size(0) == means.size(0), "covars must have the same N as means")
    _require(Ks.size(0) == viewmats.size(0), "Ks must have the same C as viewmats")


def world_to_image_projection_fwd(means, covars, viewmats, Ks, dim1, dim0, eps_blur, radius_clip):
    for n, t in (("means", means), ("covars", covars), ("viewmats", viewmats), ("Ks", Ks)):
        _check_cuda(n, t)
    _check_cameras(means, covars, viewmats, Ks)
    _require(float(radius_clip) > 0.0, "radius_clip must be positive")
    dim1 = _u32(dim1, "dim1")
    dim0 = _u32(dim0, "dim0")
    code = _dtype_code(means, "world_to_image_projection_fwd")
    _same_dtype("world_to_image_projection_fwd", means, covars, viewmats, Ks)
    C, N = viewmats.size(0), means.size(0)
    dev = means.device
    means2d = torch.empty((C, N, 2), dtype=means.dtype, device=dev)
    cov2d = torch.empty((C, N, 6), dtype=means.dtype, device=dev)
    radii = torch.zeros((C, N, 2), dtype=torch.int32, device=dev)
    if C * N:
        with torch.cuda.device(dev):
            _call("r2s_world_to_image_projection_fwd", code, _ptr(means), _ptr(covars),
                  _ptr(viewmats), _ptr(Ks), C, N, dim1, dim0, float(eps_blur),
                  float(radius_clip), _ptr(means2d), _ptr(cov2d), _ptr(radii), _stream(dev))
    return means2d, cov2d, radii


def world_to_image_projection_bwd(means, covars, viewmats, Ks, dim1, dim0, v_means2d, v_cov2d_3x3):
    for n, t in (("means", means), ("covars", covars), ("viewmats", viewmats), ("Ks", Ks),
                 ("v_means2d", v_means2d), ("v_cov2d_3x3", v_cov2d_3x3)):
        _check_cuda(n, t)
    _check_cameras(means, covars, viewmats, Ks)
    C, N = viewmats.size(0), means.size(0)
    _require(v_means2d.dim() == 3 and v_means2d.size(2) == 2, "v_means2d must be [C, N, 2]")
    _require(v_cov2d_3x3.dim() == 3 and v_cov2d_3x3.size(2) == 6, "v_cov2d_3x3 must be [C, N, 6]")
    _require(v_means2d.size(0) == C and v_means2d.size(1) == N, "v_means2d shape mismatch")
    _require(v_cov2d_3x3.size(0) == C and v_cov2d_3x3.size(1) == N, "v_cov2d_3x3 shape mismatch")
    code = _dtype_code(means, "world_to_image_projection_bwd")
    _same_dtype("world_to_image_projection_bwd", means, covars, viewmats, Ks, v_means2d, v_cov2d_3x3)
    dev = means.device
    v_means = torch.empty((N, 3), dtype=means.dtype, device=dev)
    v_covars = torch.empty((N, 6), dtype=means.dtype, device=dev)
    if N:
        with torch.cuda.device(dev):
            _call("r2s_world_to_image_projection_bwd", code, _ptr(means), _ptr(covars),
                  _ptr(viewmats), _ptr(Ks), C, N, _u32(dim1, "dim1"), _u32(dim0, "dim0"),
                  _ptr(v_means2d), _ptr(v_cov2d_3x3), _ptr(v_means), _ptr(v_covars), _stream(dev))
    return v_means, v_covars


def conics_mu_fwd(cov2d_3x3, eps):
    _check_cuda("cov2d_3x3", cov2d_3x3)
    _require(cov2d_3x3.dim() == 3, "cov2d_3x3 must be 3D [C, N, 6]")
    _require(cov2d_3x3.size(2) == 6, "cov2d_3x3 last dim must be 6")
    code = _dtype_code(cov2d_3x3, "conics_mu_fwd")
    C, N = cov2d_3x3.size(0), cov2d_3x3.size(1)
    dev = cov2d_3x3.device
    conics = torch.empty((C, N, 3), dtype=cov2d_3x3.dtype, device=dev)
    mus = torch.empty((C, N), dtype=cov2d_3x3.dtype, device=dev)
    if C * N:
        with torch.cuda.device(dev):
            _call("r2s_conics_mu_fwd", code, _ptr(cov2d_3x3), float(eps), _ptr(conics), _ptr(mus),
                  C * N, _stream(dev))
    return conics, mus


def conics_mu_bwd(cov2d_3x3, eps, conics, mus, v_conics, v_mus):
    for n, t in (("cov2d_3x3", cov2d_3x3), ("conics", conics), ("mus", mus),
                 ("v_conics", v_conics), ("v_mus", v_mus)):
        _check_cuda(n, t)
    _require(cov2d_3x3.dim() == 3, "cov2d_3x3 must be 3D [C, N, 6]")
    _require(conics.dim() == 3, "conics must be 3D [C, N, 3]")
    _require(mus.dim() == 2, "mus must be 2D [C, N]")
    _require(v_conics.dim() == 3, "v_conics must be 3D [C, N, 3]")
    _require(v_mus.dim() == 2, "v_mus must be 2D [C, N]")
    C, N = cov2d_3x3.size(0), cov2d_3x3.size(1)
    _require(cov2d_3x3.size(2) == 6, "cov2d_3x3 last dim must be 6")
    _require(tuple(conics.shape) == (C, N, 3), "conics shape must be [C, N, 3]")
    _require(tuple(mus.shape) == (C, N), "mus shape must be [C, N]")
    _require(tuple(v_conics.shape) == (C, N, 3), "v_conics shape must be [C, N, 3]")
    _require(tuple(v_mus.shape) == (C, N), "v_mus shape must be [C, N]")
    code = _dtype_code(cov2d_3x3, "conics_mu_bwd")
    _same_dtype("conics_mu_bwd", cov2d_3x3, conics, mus, v_conics, v_mus)
    dev = cov2d_3x3.device
    v_cov = torch.empty((C, N, 6), dtype=cov2d_3x3.dtype, device=dev)
    if C * N:
        with torch.cuda.device(dev):
            _call("r2s_conics_mu_bwd", code, _ptr(cov2d_3x3), float(eps), _ptr(conics), _ptr(mus),
                  _ptr(v_conics), _ptr(v_mus), _ptr(v_cov), C * N, _stream(dev))
    return v_cov


# ---------------------------------------------------------------------------
# volume mapping
# ---------------------------------------------------------------------------
def world_to_volume_mapping_fwd(means, covars, max_scales, ranges, centers, dim2, dim1, dim0,
                                eps3d, radius_clip):
    for n, t in (("means", means), ("covars", covars), ("max_scales", max_scales),
                 ("ranges", ranges), ("centers", centers)):
        _check_cuda(n, t)
    _require(means.dim() == 2 and means.size(1) == 3, "means must be [N, 3]")
    _require(covars.dim() == 2 and covars.size(1) == 6, "covars must be [N, 6]")
    _require(max_scales.dim() == 1, "max_scales must be [N]")
    _require(ranges.dim() == 1 and ranges.size(0) == 3, "ranges must be [3]")
    _require(centers.dim() == 1 and centers.size(0) == 3, "centers must be [3]")
    N = means.size(0)
    _require(covars.size(0) == N, "covars batch dim must match means")
    _require(max_scales.size(0) == N, "max_scales batch dim must match means")
    code = _dtype_code(means, "world_to_volume_mapping_fwd")
    _same_dtype("world_to_volume_mapping_fwd", means, covars, max_scales, ranges, centers)
    dev = means.device
    means3d = torch.empty((N, 3), dtype=means.dtype, device=dev)
    conics = torch.empty((N, 6), dtype=means.dtype, device=dev)
    radii = torch.empty((N, 3), dtype=torch.int32, device=dev)
    if N:
        with torch.cuda.device(dev):
            _call("r2s_world_to_volume_mapping_fwd", code, _ptr(means), _ptr(covars),
                  _ptr(max_scales), _ptr(ranges), _ptr(centers), N, _u32(dim2, "dim2"),
                  _u32(dim1, "dim1"), _u32(dim0, "dim0"), float(eps3d), float(radius_clip),
                  _ptr(means3d), _ptr(conics), _ptr(radii), _stream(dev))
    return means3d, conics, radii


def world_to_volume_mapping_bwd(means, covars, ranges, centers, dim2, dim1, dim0, eps3d,
                                v_means3d_v, v_conics):
    for n, t in (("means", means), ("covars", covars), ("ranges", ranges), ("centers", centers),
                 ("v_means3d_v", v_means3d_v), ("v_conics", v_conics)):
        _check_cuda(n, t)
    _require(means.dim() == 2 and means.size(1) == 3, "means must be [N, 3]")
    _require(covars.dim() == 2 and covars.size(1) == 6, "covars must be [N, 6]")
    _require(ranges.dim() == 1 and ranges.size(0) == 3, "ranges must be [3]")
    _require(centers.dim() == 1 and centers.size(0) == 3, "centers must be [3]")
    _require(v_means3d_v.dim() == 2 and v_means3d_v.size(1) == 3, "v_means3d_v must be [N, 3]")
    _require(v_conics.dim() == 2 and v_conics.size(1) == 6, "v_conics must be [N, 6]")
    N = means.size(0)
    _require(covars.size(0) == N, "covars shape mismatch")
    _require(v_means3d_v.size(0) == N, "v_means3d_v shape mismatch")
    _require(v_conics.size(0) == N, "v_conics shape mismatch")
    code = _dtype_code(means, "world_to_volume_mapping_bwd")
    _same_dtype("world_to_volume_mapping_bwd", means, covars, ranges, centers, v_means3d_v, v_conics)
    dev = means.device
    v_means = torch.empty((N, 3), dtype=means.dtype, device=dev)
    v_covars = torch.empty((N, 6), dtype=means.dtype, device=dev)
    if N:
        with torch.cuda.device(dev):
            _call("r2s_world_to_volume_mapping_bwd", code, _ptr(means), _ptr(covars), _ptr(ranges),
                  _ptr(centers), N, _u32(dim2, "dim2"), _u32(dim1, "dim1"), _u32(dim0, "dim0"),
                  float(eps3d), _ptr(v_means3d_v), _ptr(v_conics), _ptr(v_means), _ptr(v_covars),
                  _stream(dev))
    return v_means, v_covars


# ---------------------------------------------------------------------------
# tile binning
# ---------------------------------------------------------------------------
def isect_tiles(means2d, radii, tile_size, n_tiles_dim1, n_tiles_dim0):
    _check_cuda("means2d", means2d)
    _check_cuda("radii", radii)
    _require(means2d.dim() == 3, "means2d must be 3D [C, N, 2]")
    _require(radii.dim() == 2 or (radii.dim() == 3 and radii.size(2) == 2),
             "radii must be 2D [C, N] or 3D [C, N, 2]")
    _require(means2d.size(2) == 2, "means2d last dim must be 2")
    _require(means2d.size(0) == radii.size(0), "C dimension must match")
    _require(means2d.size(1) == radii.size(1), "N dimension must match")
    _require(radii.dtype == torch.int32, "radii must be int32")
    tile = _u32(tile_size, "tile_size")
    ntx = _u32(n_tiles_dim1, "n_tiles_dim1")
    nty = _u32(n_tiles_dim0, "n_tiles_dim0")
    code = _dtype_code(means2d, "compute_tiles_per_gauss")
    C, N = means2d.size(0), means2d.size(1)
    dev = means2d.device
    tiles_per_gauss = torch.empty((C, N), dtype=torch.int32, device=dev)
    if C * N == 0:
        return (tiles_per_gauss, torch.empty((0,), dtype=torch.int64, device=dev),
                torch.empty((0,), dtype=torch.int32, device=dev))
    T = ntx * nty
    with torch.cuda.device(dev):
        rects = torch.empty((C * N * _RECT2_BYTES,), dtype=torch.uint8, device=dev)
        ws = _bin_workspace(dev, C, N, T, 0)
        offsets = torch.empty((max(C * T, 1),), dtype=torch.int32, device=dev)
        n_dev = torch.empty((1,), dtype=torch.int64, device=dev)
        st = _stream(dev)
        _call("r2s_isect_tiles_prepare", code, _ptr(means2d), _ptr(radii),
              1 if radii.dim() == 3 else 0, C, N, tile, ntx, nty, _ptr(tiles_per_gauss),
              _ptr(rects), _ptr(ws), ws.numel(), _ptr(offsets), _ptr(n_dev), st)
        n = _read_count(n_dev)
        isect_ids = torch.empty((n,), dtype=torch.int64, device=dev)
        flatten_ids = torch.empty((n,), dtype=torch.int32, device=dev)
        if n:
            _call("r2s_bin_place", _ptr(rects), C, N, T, ntx, 0, 0, _ptr(ws), ws.numel(),
                  _ptr(offsets), n, _ptr(flatten_ids), _ptr(isect_ids), st)
    return tiles_per_gauss, isect_ids, flatten_ids


def isect_offset_encode(isect_ids, C, n_tiles_dim1, n_tiles_dim0):
    _check_cuda("isect_ids", isect_ids)
    _require(isect_ids.dtype == torch.int64, "isect_ids must be int64")
    C = _u32(C, "C")
    ntx = _u32(n_tiles_dim1, "n_tiles_dim1")
    nty = _u32(n_tiles_dim0, "n_tiles_dim0")
    dev = isect_ids.device
    offsets = torch.empty((C, nty, ntx), dtype=torch.int32, device=dev)
    n = isect_ids.numel()
    if n == 0:
        offsets.fill_(0)
        return offsets
    if offsets.numel():
        with torch.cuda.device(dev):
            _call("r2s_isect_offset_encode", _ptr(isect_ids), n, offsets.numel(), _ptr(offsets),
                  _stream(dev))
    return offsets


def isect_tiles_3d(means3d, radii, tile_size, n_tiles_dim2, n_tiles_dim1, n_tiles_dim0):
    _check_cuda("means3d", means3d)
    _check_cuda("radii", radii)
    _require(means3d.dim() == 2, "means3d must be 2D [N, 3]")
    _require(radii.dim() == 2, "radii must be 2D [N, 3]")
    _require(means3d.size(1) == 3, "means3d last dim must be 3")
    _require(radii.size(1) == 3, "radii last dim must be 3")
    _require(means3d.size(0) == radii.size(0), "N dimension must match")
    _require(radii.dtype == torch.int32, "radii must be int32")
    tile = _u32(tile_size, "tile_size")
    nt2 = _u32(n_tiles_dim2, "n_tiles_dim2")
    nt1 = _u32(n_tiles_dim1, "n_tiles_dim1")
    nt0 = _u32(n_tiles_dim0, "n_tiles_dim0")
    code = _dtype_code(means3d, "compute_tiles_per_gauss_3d")
    N = means3d.size(0)
    dev = means3d.device
    tiles_per_gauss = torch.empty((N,), dtype=torch.int32, device=dev)
    if N == 0:
        return (tiles_per_gauss, torch.empty((0,), dtype=torch.int64, device=dev),
                torch.empty((0,), dtype=torch.int32, device=dev))
    T = nt1 * nt2
    with torch.cuda.device(dev):
        rects = torch.empty((N * _RECT3_BYTES,), dtype=torch.uint8, device=dev)
        ws = _bin_workspace(dev, nt0, N, T, 1)
        offsets = torch.empty((max(nt0 * T, 1),), dtype=torch.int32, device=dev)
        n_dev = torch.empty((1,), dtype=torch.int64, device=dev)
        st = _stream(dev)
        _call("r2s_isect_tiles_3d_prepare", code, _ptr(means3d), _ptr(radii), N, tile, nt2, nt1,
              nt0, _ptr(tiles_per_gauss), _ptr(rects), _ptr(ws), ws.numel(), _ptr(offsets),
              _ptr(n_dev), st)
        n = _read_count(n_dev)
        isect_ids = torch.empty((n,), dtype=torch.int64, device=dev)
        flatten_ids = torch.empty((n,), dtype=torch.int32, device=dev)
        if n:
            _call("r2s_bin_place", _ptr(rects), nt0, N, T, nt2, 1, 0, _ptr(ws), ws.numel(),
                  _ptr(offsets), n, _ptr(flatten_ids), _ptr(isect_ids), st)
    return tiles_per_gauss, isect_ids, flatten_ids


def isect_offset_encode_3d(isect_ids, n_tiles_dim2, n_tiles_dim1, n_tiles_dim0):
    _check_cuda("isect_ids", isect_ids)
    _require(isect_ids.dtype == torch.int64, "isect_ids must be int64")
    nt2 = _u32(n_tiles_dim2, "n_tiles_dim2")
    nt1 = _u32(n_tiles_dim1, "n_tiles_dim1")
    nt0 = _u32(n_tiles_dim0, "n_tiles_dim0")
    dev = isect_ids.device
    offsets = torch.empty((nt0, nt1, nt2), dtype=torch.int32, device=dev)
    n = isect_ids.numel()
    if n == 0:
        offsets.fill_(0)
        return offsets
    if offsets.numel():
        with torch.cuda.device(dev):
            _call("r2s_isect_offset_encode", _ptr(isect_ids), n, offsets.numel(), _ptr(offsets),
                  _stream(dev))
    return offsets


# ---------------------------------------------------------------------------
# rasterization
# ---------------------------------------------------------------------------
def _check_raster_inputs(means2d, conics, opacities, mus, tile_offsets, flatten_ids):
    for n, t in (("means2d", means2d), ("conics", conics), ("opacities", opacities),
                 ("mus", mus), ("tile_offsets", tile_offsets), ("flatten_ids", flatten_ids)):
        _check_cuda(n, t)
    _require(means2d.dim() == 3, "means2d must be 3D [C, N, 2]")
    _require(conics.dim() == 3, "conics must be 3D [C, N, 3]")
    _require(opacities.dim() == 2, "opacities must be 2D [C, N]")
    _require(mus.dim() == 2, "mus must be 2D [C, N]")
    _require(tile_offsets.dim() == 3, "tile_offsets must be 3D [C, n_tiles_dim0, n_tiles_dim1]")
    _require(flatten_ids.dim() == 1, "flatten_ids must be 1D [n_isects]")
    _require(means2d.size(2) == 2, "means2d last dim must be 2")
    _require(conics.size(2) == 3, "conics last dim must be 3")
    C, N = means2d.size(0), means2d.size(1)
    _require(conics.size(0) == C and conics.size(1) == N, "conics shape must match means2d [C, N, 3]")
    _require(opacities.size(0) == C and opacities.size(1) == N, "opacities shape must match [C, N]")
    _require(mus.size(0) == C and mus.size(1) == N, "mus shape must match [C, N]")
    _require(tile_offsets.size(0) == C, "tile_offsets C dimension must match")
    _require(tile_offsets.dtype == torch.int32, "tile_offsets must be int32")
    _require(flatten_ids.dtype == torch.int32, "flatten_ids must be int32")
    _same_dtype("rasterize_to_pixels", means2d, conics, opacities, mus)
    return C, N


def _splat_scratch(means2d, C, N, tile):
    """Packed splat records for the float32 16-pixel-tile kernels (else None)."""
    if means2d.dtype == torch.float32 and int(tile) == 16:
        return torch.empty((C * N * 8,), dtype=torch.float32, device=means2d.device)
    return None


def rasterize_to_pixels_fwd(means2d, conics, opacities, mus, tile_offsets, flatten_ids, dim1,
                            dim0, tile_size):
    C, N = _check_raster_inputs(means2d, conics, opacities, mus, tile_offsets, flatten_ids)
    code = _dtype_code(means2d, "rasterize_to_pixels_fwd")
    W = _u32(dim1, "dim1")
    H = _u32(dim0, "dim0")
    tile = _u32(tile_size, "tile_size")
    nty, ntx = tile_offsets.size(1), tile_offsets.size(2)
    dev = means2d.device
    out = torch.empty((C, H, W), dtype=means2d.dtype, device=dev)
    n = flatten_ids.size(0)
    if C == 0 or N == 0 or n == 0:
        out.zero_()
        return out
    with torch.cuda.device(dev):
        scratch = _splat_scratch(means2d, C, N, tile)
        _call("r2s_rasterize_to_pixels_fwd", code, _ptr(means2d), _ptr(conics), _ptr(opacities),
              _ptr(mus), _ptr(tile_offsets), _ptr(flatten_ids), C, N, n, W, H, tile, ntx, nty,
              _ptr(scratch), _ptr(out), _stream(dev))
    return out


def _raster_bwd(mode, means2d, conics, opacities, mus, tile_offsets, flatten_ids, v_render_output,
                dim1, dim0, tile_size, absgrad):
    C, N = _check_raster_inputs(means2d, conics, opacities, mus, tile_offsets, flatten_ids)
    _check_cuda("v_render_output", v_render_output)
    W = _u32(dim1, "dim1")
    H = _u32(dim0, "dim0")
    tile = _u32(tile_size, "tile_size")
    _require(v_render_output.dim() == 3, "v_render_output must be 3D [C, dim0, dim1]")
    _require(v_render_output.size(0) == C and v_render_output.size(1) == H
             and v_render_output.size(2) == W, "v_render_output shape must be [C, dim0, dim1]")
    code = _dtype_code(means2d, "rasterize_to_pixels_bwd")
    _same_dtype("rasterize_to_pixels_bwd", means2d, v_render_output)
    dev = means2d.device
    v_means2d = torch.zeros_like(means2d)
    v_abs = torch.zeros_like(means2d) if absgrad else None
    v_conics = torch.zeros_like(conics)
    v_opac = torch.zeros_like(opacities)
    v_mus = torch.zeros_like(mus)
    n = flatten_ids.size(0)
    if C == 0 or N == 0 or n == 0:
        return v_abs, v_means2d, v_conics, v_opac, v_mus
    nty, ntx = tile_offsets.size(1), tile_offsets.size(2)
    with torch.cuda.device(dev):
        stats = torch.empty((C * N * 8,), dtype=means2d.dtype, device=dev)
        scratch = _splat_scratch(means2d, C, N, tile)
        _call("r2s_rasterize_to_pixels_bwd", code, mode, _ptr(means2d), _ptr(conics),
              _ptr(opacities), _ptr(mus), _ptr(tile_offsets), _ptr(flatten_ids),
              _ptr(v_render_output), C, N, n, W, H, tile, ntx, nty, _ptr(scratch), _ptr(stats),
              _ptr(v_abs),
              _ptr(v_means2d), _ptr(v_conics), _ptr(v_opac), _ptr(v_mus), _stream(dev))
    return v_abs, v_means2d, v_conics, v_opac, v_mus


def rasterize_to_pixels_bwd(means2d, conics, opacities, mus, tile_offsets, flatten_ids,
                            v_render_output, dim1, dim0, tile_size, absgrad):
    return _raster_bwd(0, means2d, conics, opacities, mus, tile_offsets, flatten_ids,
                       v_render_output, dim1, dim0, tile_size, absgrad)


def rasterize_to_pixels_bwd_per_gaussian(means2d, conics, opacities, mus, tile_offsets, isect_ids,
                                         flatten_ids, v_render_output, dim1, dim0, tile_size,
                                         absgrad):
    _check_cuda("isect_ids", isect_ids)
    _require(isect_ids.dim() == 1, "isect_ids must be 1D [n_isects]")
    _require(isect_ids.dtype == torch.int64, "isect_ids must be int64")
    _require(isect_ids.size(0) == flatten_ids.size(0),
             "isect_ids and flatten_ids must have the same length")
    return _raster_bwd(1, means2d, conics, opacities, mus, tile_offsets, flatten_ids,
                       v_render_output, dim1, dim0, tile_size, absgrad)


# ---------------------------------------------------------------------------
# voxelization
# ---------------------------------------------------------------------------
def _check_voxel_inputs(means3d, conics, opacities, tile_offsets, flatten_ids):
    for n, t in (("means3d", means3d), ("conics", conics), ("opacities", opacities),
                 ("tile_offsets", tile_offsets), ("flatten_ids", flatten_ids)):
        _check_cuda(n, t)
    _require(means3d.dim() == 2, "means3d must be 2D [N, 3]")
    _require(conics.dim() == 2, "conics must be 2D [N, 6]")
    _require(opacities.dim() == 1, "opacities must be 1D [N]")
    _require(tile_offsets.dim() == 3,
             "tile_offsets must be 3D [n_tiles_dim0, n_tiles_dim1, n_tiles_dim2]")
    _require(flatten_ids.dim() == 1, "flatten_ids must be 1D [n_isects]")
    _require(means3d.size(1) == 3, "means3d last dim must be 3")
    _require(conics.size(1) == 6, "conics last dim must be 6")
    N = means3d.size(0)
    _require(conics.size(0) == N, "conics first dim must match N")
    _require(opacities.size(0) == N, "opacities first dim must match N")
    _require(tile_offsets.dtype == torch.int32, "tile_offsets must be int32")
    _require(flatten_ids.dtype == torch.int32, "flatten_ids must be int32")
    _same_dtype("voxelize_to_voxels", means3d, conics, opacities)
    return N


def voxelize_to_voxels_fwd(means3d, conics, opacities, tile_offsets, flatten_ids, dim2, dim1, dim0,
                           tile_size):
    N = _check_voxel_inputs(means3d, conics, opacities, tile_offsets, flatten_ids)
    code = _dtype_code(means3d, "voxelize_to_voxels_fwd")
    d2, d1, d0 = _u32(dim2, "dim2"), _u32(dim1, "dim1"), _u32(dim0, "dim0")
    tile = _u32(tile_size, "tile_size")
    nt0, nt1, nt2 = tile_offsets.size(0), tile_offsets.size(1), tile_offsets.size(2)
    dev = means3d.device
    out = torch.zeros((d0, d1, d2), dtype=means3d.dtype, device=dev)
    n = flatten_ids.size(0)
    if N == 0 or n == 0 or out.numel() == 0:
        return out
    with torch.cuda.device(dev):
        _call("r2s_voxelize_to_voxels_fwd", code, _ptr(means3d), _ptr(conics), _ptr(opacities),
              _ptr(tile_offsets), _ptr(flatten_ids), N, n, d2, d1, d0, tile, nt2, nt1, nt0,
              _ptr(out), _stream(dev))
    return out


def _voxel_bwd(mode, means3d, conics, opacities, tile_offsets, flatten_ids, v_render_output, dim2,
               dim1, dim0, tile_size):
    N = _check_voxel_inputs(means3d, conics, opacities, tile_offsets, flatten_ids)
    _check_cuda("v_render_output", v_render_output)
    _require(v_render_output.dim() == 3, "v_render_output must be 3D [dim0, dim1, dim2]")
    d2, d1, d0 = _u32(dim2, "dim2"), _u32(dim1, "dim1"), _u32(dim0, "dim0")
    _require(tuple(v_render_output.shape) == (d0, d1, d2),
             "v_render_output shape must be [dim0, dim1, dim2]")
    code = _dtype_code(means3d, "voxelize_to_voxels_bwd")
    _same_dtype("voxelize_to_voxels_bwd", means3d, v_render_output)
    tile = _u32(tile_size, "tile_size")
    dev = means3d.device
    v_means3d = torch.zeros_like(means3d)
    v_conics = torch.zeros_like(conics)
    v_opac = torch.zeros_like(opacities)
    n = flatten_ids.size(0)
    if N == 0 or n == 0:
        return v_means3d, v_conics, v_opac
    nt0, nt1, nt2 = tile_offsets.size(0), tile_offsets.size(1), tile_offsets.size(2)
    with torch.cuda.device(dev):
        stats = torch.empty((N * 12,), dtype=means3d.dtype, device=dev)
        _call("r2s_voxelize_to_voxels_bwd", code, mode, _ptr(means3d), _ptr(conics),
              _ptr(opacities), _ptr(tile_offsets), _ptr(flatten_ids), _ptr(v_render_output), N, n,
              d2, d1, d0, tile, nt2, nt1, nt0, _ptr(stats), _ptr(v_means3d), _ptr(v_conics),
              _ptr(v_opac), _stream(dev))
    return v_means3d, v_conics, v_opac


def voxelize_to_voxels_bwd(means3d, conics, opacities, tile_offsets, flatten_ids, v_render_output,
                           dim2, dim1, dim0, tile_size):
    return _voxel_bwd(0, means3d, conics, opacities, tile_offsets, flatten_ids, v_render_output,
                      dim2, dim1, dim0, tile_size)


def voxelize_to_voxels_bwd_per_gaussian(means3d, conics, opacities, tile_offsets, isect_ids,
                                        flatten_ids, v_render_output, dim2, dim1, dim0, tile_size):
    _check_cuda("isect_ids", isect_ids)
    _require(isect_ids.dim() == 1, "isect_ids must be 1D")
    _require(isect_ids.dtype == torch.int64, "isect_ids must be int64")
    _require(isect_ids.size(0) == flatten_ids.size(0),
             "isect_ids and flatten_ids must have the same length")
    return _voxel_bwd(1, means3d, conics, opacities, tile_offsets, flatten_ids, v_render_output,
                      dim2, dim1, dim0, tile_size)


# ---------------------------------------------------------------------------
# fused float32 helpers for r2splat.ops (not part of the reference API)
# ---------------------------------------------------------------------------
def fused_prepare(quats, raw_scales, raw_opacities, scale_min, scale_max):
    N = quats.size(0)
    dev = quats.device
    covars = torch.empty((N, 6), dtype=torch.float32, device=dev)
    max_scales = torch.empty((N,), dtype=torch.float32, device=dev)
    opac = torch.empty((N,), dtype=torch.float32, device=dev)
    if N:
        _call("r2s_prepare_gaussians_f32", _ptr(quats), _ptr(raw_scales), _ptr(raw_opacities),
              float(scale_min), float(scale_max), _ptr(covars), _ptr(max_scales), _ptr(opac), N,
              _stream(dev))
    return covars, max_scales, opac


def fused_project(means, covars, opacities, viewmats, Ks, W, H, tile, ntx, nty, eps2d, clip,
                  want_counts=False):
    C, N = viewmats.size(0), means.size(0)
    dev = means.device
    means2d = torch.empty((C, N, 2), dtype=torch.float32, device=dev)
    radii = torch.empty((C, N, 2), dtype=torch.int32, device=dev)
    splats = torch.empty((C, N, 8), dtype=torch.float32, device=dev)
    rects = torch.empty((C * N * _RECT2_BYTES,), dtype=torch.uint8, device=dev)
    counts = torch.empty((C, N), dtype=torch.int32, device=dev) if want_counts else None
    if C * N:
        _call("r2s_project_splats_f32", _ptr(means), _ptr(covars), _ptr(opacities),
              _ptr(viewmats), _ptr(Ks), C, N, W, H, tile, ntx, nty, float(eps2d), float(clip),
              _ptr(means2d), _ptr(radii), _ptr(splats), _ptr(rects), _ptr(counts), _stream(dev))
    return means2d, radii, splats, rects, counts


def fused_bin(rects, S, N, T, tiles_x, layered, want_keys=False, segment_base=0, limit=None):
    """Binning from precomputed rectangles -> (tile_offsets [S*T], flatten_ids,
    isect_ids or None).  With ``limit``, returns None instead when the record
    count exceeds it (the caller then bins in smaller batches)."""
    dev = rects.device
    st = _stream(dev)
    ws = _bin_workspace(dev, S, N, T, layered)
    offsets = torch.empty((max(S * T, 1),), dtype=torch.int32, device=dev)
    n_dev = torch.empty((1,), dtype=torch.int64, device=dev)
    _call("r2s_bin_prepare", _ptr(rects), S, N, T, tiles_x, layered, segment_base, _ptr(ws),
          ws.numel(), _ptr(offsets), _ptr(n_dev), st)
    n = _read_count(n_dev)
    if limit is not None and n > limit:
        return None
    flatten_ids = torch.empty((n,), dtype=torch.int32, device=dev)
    isect_ids = torch.empty((n,), dtype=torch.int64, device=dev) if want_keys else None
    if n:
        _call("r2s_bin_place", _ptr(rects), S, N, T, tiles_x, layered, segment_base, _ptr(ws),
              ws.numel(), _ptr(offsets), n, _ptr(flatten_ids), _ptr(isect_ids), st)
    return offsets[: S * T], flatten_ids, isect_ids


def fused_raster_fwd(splats, offsets, flatten_ids, C, N, W, H, tile, ntx, nty, out=None,
                     cull=None):
    """``cull``: an int16 [n_isects] tensor that receives the records'
    culling ranges (16-pixel tiles only), or None."""
    dev = splats.device
    if out is None:
        out = torch.empty((C, H, W), dtype=torch.float32, device=dev)
    _call("r2s_raster_splats_fwd_f32", _ptr(splats), _ptr(offsets), _ptr(flatten_ids), C, N,
          flatten_ids.numel(), W, H, tile, ntx, nty, _ptr(out), _ptr(cull), _stream(dev))
    return out


def fused_raster_bwd(splats, offsets, flatten_ids, v_image, C, N, W, H, tile, ntx, nty, with_abs,
                     out=None, cull=None):
    """``cull``: the table fused_raster_fwd wrote for the same binning, or None."""
    dev = splats.device
    stats = torch.empty((C * N, 8), dtype=torch.float32, device=dev) if out is None else out
    _call("r2s_raster_splats_bwd_f32", _ptr(splats), _ptr(offsets), _ptr(flatten_ids),
          _ptr(v_image), C, N, flatten_ids.numel(), W, H, tile, ntx, nty, 1 if with_abs else 0,
          _ptr(cull), _ptr(stats), _stream(dev))
    return stats


# Largest number of intersection records one binning holds: tile offsets and
# flatten ids are int32, as in the reference (IsectTiles.cpp:95-107).
MAX_RECORDS_PER_BATCH = 2 ** 31 - 1


def plan_view_batches(rects, C, N, max_records=None):
    """Contiguous view ranges [(c0, c1)] whose records each fit one binning
    (views of more records than the limit get a batch of their own, which the
    binning then rejects).  rects: the [C*N] packed tile rectangles."""
    limit = MAX_RECORDS_PER_BATCH if max_records is None else int(max_records)
    r = rects.view(torch.int32).view(C, N, 2).to(torch.int64) & 0xFFFFFFFF
    w = ((r[..., 0] >> 16) - (r[..., 0] & 0xFFFF)).clamp_min(0)
    h = ((r[..., 1] >> 16) - (r[..., 1] & 0xFFFF)).clamp_min(0)
    per_view = (w * h).sum(dim=1).tolist()
    batches, c0, acc = [], 0, 0
    for c, n in enumerate(per_view):
        if c > c0 and acc + n > limit:
            batches.append((c0, c))
            c0, acc = c, 0
        acc += n
    if C > c0:
        batches.append((c0, C))
    return batches


def fused_map(means, covars, opacities, ranges, centers, dim2, dim1, dim0, tile, nt2, nt1, nt0,
              eps3d, clip, want_counts=False):
    N = means.size(0)
    dev = means.device
    means3d = torch.empty((N, 3), dtype=torch.float32, device=dev)
    conics = torch.empty((N, 6), dtype=torch.float32, device=dev)
    radii = torch.empty((N, 3), dtype=torch.int32, device=dev)
    vsplats = torch.empty((N, 16), dtype=torch.float32, device=dev)
    rects = torch.empty((N * _RECT3_BYTES,), dtype=torch.uint8, device=dev)
    counts = torch.empty((N,), dtype=torch.int32, device=dev) if want_counts else None
    if N:
        _call("r2s_map_vsplats_f32", _ptr(means), _ptr(covars), _ptr(opacities), _ptr(ranges),
              _ptr(centers), N, dim2, dim1, dim0, tile, nt2, nt1, nt0, float(eps3d), float(clip),
              _ptr(means3d), _ptr(conics), _ptr(radii), _ptr(vsplats), _ptr(rects), _ptr(counts),
              _stream(dev))
    return means3d, conics, radii, vsplats, rects, counts


def fused_brick_order(offsets, n_isects):
    """Longest-first launch order [n_keys] (int32) of the bricks of a 3D
    binning (``r2s_brick_order``)."""
    dev = offsets.device
    order = torch.empty((offsets.numel(),), dtype=torch.int32, device=dev)
    _call("r2s_brick_order", _ptr(offsets), offsets.numel(), int(n_isects), _ptr(order),
          _stream(dev))
    return order


def fused_voxel_rows(vsplats, offsets, flatten_ids, N, dim2, dim1, dim0, tile, nt2, nt1, nt0,
                     layer_begin=0, layer_end=None, order=None):
    """Row table [n_isects, 2] (int32 bit patterns) of a 3D binning with
    8-voxel bricks, or None for other brick sizes."""
    if tile != 8:
        return None
    dev = vsplats.device
    if layer_end is None:
        layer_end = nt0
    rows = torch.empty((flatten_ids.numel(), 2), dtype=torch.int32, device=dev)
    _call("r2s_voxel_rows_f32", _ptr(vsplats), _ptr(offsets), _ptr(flatten_ids), N,
          flatten_ids.numel(), dim2, dim1, dim0, tile, nt2, nt1, nt0, layer_begin, layer_end,
          _ptr(order), _ptr(rows), _stream(dev))
    return rows


def fused_voxel_fwd(vsplats, offsets, flatten_ids, N, dim2, dim1, dim0, tile, nt2, nt1, nt0,
                    layer_begin=0, layer_end=None, out=None, rows=None, order=None):
    dev = vsplats.device
    if layer_end is None:
        layer_end = nt0
    z0 = layer_begin * tile
    z1 = min(layer_end * tile, dim0)
    if out is None:
        out = torch.empty((max(z1 - z0, 0), dim1, dim2), dtype=torch.float32, device=dev)
    _call("r2s_voxel_splats_fwd_f32", _ptr(vsplats), _ptr(offsets), _ptr(flatten_ids), _ptr(rows),
          N, flatten_ids.numel(), dim2, dim1, dim0, tile, nt2, nt1, nt0, layer_begin, layer_end,
          _ptr(order), _ptr(out), _stream(dev))
    return out


def fused_voxel_bwd(vsplats, offsets, flatten_ids, v_volume, N, dim2, dim1, dim0, tile, nt2, nt1,
                    nt0, layer_begin=0, layer_end=None, rows=None, order=None):
    """Voxel backward statistics [N, 12], float64 per-Gaussian sums
    (r2s_voxel_splats_bwd_f32), the input of fused_explicit_backward."""
    dev = vsplats.device
    if layer_end is None:
        layer_end = nt0
    stats = torch.empty((N, 12), dtype=torch.float64, device=dev)
    _call("r2s_voxel_splats_bwd_f32", _ptr(vsplats), _ptr(offsets), _ptr(flatten_ids), _ptr(rows),
          _ptr(v_volume), N, flatten_ids.numel(), dim2, dim1, dim0, tile, nt2, nt1, nt0,
          layer_begin, layer_end, _ptr(order), _ptr(stats), _stream(dev))
    return stats


def fused_explicit_backward(means, quats, raw_scales, raw_opacities, scale_min, scale_max,
                            viewmats, Ks, W, H, eps2d, raster_stats, v_means2d, v_means2d_abs,
                            ranges, centers, dim2, dim1, dim0, eps3d, vox_stats, accumulate, outs,
                            densify=None):
    """``densify``: None, or (radii [C,N,2] int32, scale_x, scale_y, extent,
    absgrad, grad2d [N], count [N], max_radii [N] or None) for the fused
    densification statistics.  ``vox_stats``: the float64 output of
    fused_voxel_bwd, or None."""
    _require(vox_stats is None or vox_stats.dtype == torch.float64,
             "vox_stats must be the float64 statistics of fused_voxel_bwd")
    dev = means.device
    C = 0 if viewmats is None else viewmats.size(0)
    N = means.size(0)
    v_means, v_quats, v_scales, v_opac = outs
    args = (_ptr(means), _ptr(quats), _ptr(raw_scales), _ptr(raw_opacities), float(scale_min),
            float(scale_max), _ptr(viewmats), _ptr(Ks), C, N, W, H, float(eps2d),
            _ptr(raster_stats), _ptr(v_means2d), _ptr(v_means2d_abs), _ptr(ranges),
            _ptr(centers), dim2, dim1, dim0, float(eps3d), _ptr(vox_stats),
            1 if accumulate else 0, _ptr(v_means), _ptr(v_quats), _ptr(v_scales), _ptr(v_opac))
    if densify is None:
        _call("r2s_explicit_backward_f32", *args, _stream(dev))
        return
    radii, sx, sy, extent, absgrad, grad2d, count, max_radii = densify
    from ._backend import DensifyArgs
    d = DensifyArgs(_ptr(radii), float(sx), float(sy), float(extent), 1 if absgrad else 0,
                    _ptr(grad2d), _ptr(count), _ptr(max_radii))
    _call("r2s_explicit_backward_densify_f32", *args, ctypes.byref(d), _stream(dev))


def is_cuda_extension_available() -> bool:
    try:
        return is_cuda_available()
    except ImportError:
        return False


__all__ = [
    "isect_tiles",
    "parameter_transform_fwd",
    "parameter_transform_bwd",
    "isect_offset_encode",
    "isect_tiles_3d",
    "isect_offset_encode_3d",
    "conics_mu_fwd",
    "conics_mu_bwd",
    "world_to_image_projection_fwd",
    "world_to_image_projection_bwd",
    "world_to_volume_mapping_fwd",
    "world_to_volume_mapping_bwd",
    "rasterize_to_pixels_fwd",
    "rasterize_to_pixels_bwd",
    "rasterize_to_pixels_bwd_per_gaussian",
    "voxelize_to_voxels_fwd",
    "voxelize_to_voxels_bwd",
    "voxelize_to_voxels_bwd_per_gaussian",
    "is_cuda_extension_available",
]
