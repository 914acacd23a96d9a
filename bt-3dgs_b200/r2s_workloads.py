"""Seeded synthetic workloads of the benchmark configurations.

The reference ships no dataset for this path; the configurations below are
the synthetic stand-ins (Gaussian counts, scale and density distributions,
orbit and detector sizes, voxel grids).  Geometry restates the reference's
cone-beam data loader (src/data/ctproj.py:137-267): focal length
DSD * n / span, principal point at the detector centre, camera-to-world
Rz(theta) @ R_base with R_base = [[0,0,-1],[1,0,0],[0,-1,0]] and the source
at (DSO cos theta, DSO sin theta, 0); the view matrix is the rigid inverse
(src/utils/math.py:5-32).  Raw parameters invert the model's activations:
scales through the bounded sigmoid (src/models/gaussian_model.py:266-274)
and densities through softplus (gaussian_model.py:680-684).

Everything is generated on the CPU (numpy PCG64, float64, then float32) and
moved by the caller.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import numpy as np
import torch

SCALE_MIN = 5e-4  # configs/model/binary_tree.yaml:6
SCALE_MAX = 1.0  # configs/model/binary_tree.yaml:7
EPS2D = 1e-8  # configs/model/binary_tree.yaml:10
EPS3D = 1e-8  # configs/model/binary_tree.yaml:11
IMG_TILE = 16  # configs/model/binary_tree.yaml:12
VOL_TILE = 8  # configs/model/binary_tree.yaml:13
RADIUS_CLIP = 3.0  # configs/model/binary_tree.yaml:14-15
DSO = 2.0
DSD = 3.0
DETECTOR_SPAN = 1.5


@dataclass(frozen=True)
class WorkloadConfig:
    name: str
    n_gaussians: int
    n_views: int
    detector: int
    grid: int
    log_scale_lo: float
    log_scale_hi: float
    means: str  # "uniform", "clusters", "shell"
    density: str  # "uniform", "lognormal"
    seed: int = 0


CONFIGS: Dict[int, WorkloadConfig] = {
    0: WorkloadConfig("cfg0-1k-1view-128px-64vox", 1024, 1, 128, 64,
                      math.log(0.005), math.log(0.05), "uniform", "uniform", 0),
    1: WorkloadConfig("cfg1-50k-50views-256px-128vox", 50_000, 50, 256, 128,
                      math.log(0.005), math.log(0.05), "clusters", "uniform", 1),
    2: WorkloadConfig("cfg2-500k-75views-512px-256vox", 500_000, 75, 512, 256,
                      math.log(0.002), math.log(0.03), "clusters", "lognormal", 2),
    3: WorkloadConfig("cfg3-2M-shell-100views-768px-512vox", 2_000_000, 100, 768, 512,
                      math.log(0.005), math.log(0.05), "shell", "uniform", 3),
    4: WorkloadConfig("cfg4-1M-train-8views-512px-64vox", 1_000_000, 8, 512, 64,
                      math.log(0.005), math.log(0.05), "uniform", "uniform", 4),
}


def inverse_scale(s: torch.Tensor, smin: float = SCALE_MIN, smax: float = SCALE_MAX) -> torch.Tensor:
    eps = 1e-5
    s = s.clamp(min=smin + eps, max=smax - eps)
    p = ((s - smin) / (smax - smin)).clamp(1e-6, 1 - 1e-6)
    return torch.logit(p)


def inverse_softplus(rho: torch.Tensor) -> torch.Tensor:
    rho = rho.clamp_min(1e-6)
    return torch.where(rho > 20, rho, torch.log(torch.expm1(rho)))


def _means(cfg: WorkloadConfig, n: int, g: np.random.Generator) -> np.ndarray:
    if cfg.means == "uniform":
        return g.random((n, 3)) - 0.5
    if cfg.means == "clusters":
        centers = (g.random((8, 3)) - 0.5) * 0.7
        which = g.integers(0, 8, n)
        m = centers[which] + 0.12 * g.standard_normal((n, 3))
        return np.clip(m, -0.5, 0.5)
    if cfg.means == "shell":
        n_shell = int(round(0.3 * n))
        cube = g.random((n - n_shell, 3)) - 0.5
        d = g.standard_normal((n_shell, 3))
        d = d / np.maximum(np.linalg.norm(d, axis=-1, keepdims=True), 1e-12)
        r = 0.39 + 0.02 * g.random((n_shell, 1))
        m = np.concatenate((cube, d * r), 0)
        return m[g.permutation(n)]
    raise ValueError(cfg.means)


def make_gaussians(cfg: WorkloadConfig, n: Optional[int] = None, seed: Optional[int] = None):
    """Raw parameters (means, quats, raw_scales, raw_opacities), float32 CPU.

    Drawn with numpy's PCG64 generator in float64 (the same values on every
    machine), activations inverted in float64, then rounded to float32."""
    n = cfg.n_gaussians if n is None else int(n)
    g = np.random.default_rng(cfg.seed if seed is None else seed)
    means = _means(cfg, n, g)
    log_s = cfg.log_scale_lo + (cfg.log_scale_hi - cfg.log_scale_lo) * g.random((n, 3))
    scales = torch.from_numpy(np.exp(log_s))
    quats = g.standard_normal((n, 4))
    quats = quats / np.maximum(np.linalg.norm(quats, axis=-1, keepdims=True), 1e-12)
    if cfg.density == "uniform":
        rho = torch.from_numpy(g.random(n))
    else:
        rho = torch.from_numpy(np.exp(-2.0 + 1.0 * g.standard_normal(n)))
    return (torch.from_numpy(means).float().contiguous(), torch.from_numpy(quats).float().contiguous(),
            inverse_scale(scales).float().contiguous(), inverse_softplus(rho).float().contiguous())


def camtoworld(theta: float) -> torch.Tensor:
    base = torch.tensor([[0.0, 0.0, -1.0], [1.0, 0.0, 0.0], [0.0, -1.0, 0.0]], dtype=torch.float64)
    c, s = math.cos(theta), math.sin(theta)
    rz = torch.tensor([[c, -s, 0.0], [s, c, 0.0], [0.0, 0.0, 1.0]], dtype=torch.float64)
    T = torch.eye(4, dtype=torch.float64)
    T[:3, :3] = rz @ base
    T[:3, 3] = torch.tensor([DSO * c, DSO * s, 0.0], dtype=torch.float64)
    return T


def invert_rigid(T: torch.Tensor) -> torch.Tensor:
    Rt = T[..., :3, :3].transpose(-1, -2)
    t = T[..., :3, 3:]
    out = torch.zeros_like(T)
    out[..., :3, :3] = Rt
    out[..., :3, 3:] = -Rt @ t
    out[..., 3, 3] = 1
    return out


def make_cameras(n_views: int, detector: int, first: int = 0, count: Optional[int] = None,
                 total: Optional[int] = None, stride: int = 1):
    """viewmats [C,4,4] and Ks [C,3,3] (float32) for views first,
    first + stride, ... (count of them) of `total` views evenly spaced over 360
    degrees."""
    total = n_views if total is None else total
    count = n_views if count is None else count
    thetas = [2 * math.pi * (first + k * stride) / total for k in range(count)]
    c2w = torch.stack([camtoworld(t) for t in thetas]) if thetas else torch.zeros(0, 4, 4, dtype=torch.float64)
    viewmats = invert_rigid(c2w).float().contiguous()
    f = DSD * detector / DETECTOR_SPAN
    K = torch.tensor([[f, 0.0, detector / 2.0], [0.0, f, detector / 2.0], [0.0, 0.0, 1.0]])
    Ks = K.expand(count, 3, 3).contiguous()
    return viewmats, Ks


def unit_cube_box():
    """ranges and centers of the voxelized region [-0.5, 0.5]^3."""
    return torch.ones(3), torch.zeros(3)


__all__ = [name for name in globals() if not name.startswith("_")]
