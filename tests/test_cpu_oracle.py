"""The CPU oracle pinned against the reference suite's golden vectors, and the
binning restatement's semantics (stable order, offsets) -- no GPU needed."""
import math

import numpy as np
import pytest
import torch

from _helpers import load_golden, rel_l2
from oracle import r2s_oracle as O


@pytest.fixture(scope="module")
def golden():
    return load_golden()


def test_parameter_transform_matches_golden(golden):
    g = golden["param"]
    q = g["quats"].clone().requires_grad_(True)
    s = g["raw_scales"].clone().requires_grad_(True)
    cov, ms = O.parameter_transform(q, s, g["scale_min"], g["scale_max"])
    torch.testing.assert_close(cov.detach(), g["covars"], atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(ms.detach(), g["max_scales"], atol=1e-7, rtol=1e-6)
    gq, gs = torch.autograd.grad((cov * g["v_covars"]).sum(), (q, s))
    torch.testing.assert_close(gq, g["v_quats"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(gs, g["v_raw_scales"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("case", range(4))
def test_conics_mu_matches_golden(golden, case):
    g = golden["conics_mu"][case]
    cov = g["covars"].clone().requires_grad_(True)
    conics, mus = O.conics_mu(cov, g["eps"])
    torch.testing.assert_close(conics.detach(), g["conics"], atol=1e-12, rtol=1e-9)
    torch.testing.assert_close(mus.detach(), g["mus"], atol=1e-12, rtol=1e-9)
    grad = torch.autograd.grad((conics * g["v_conics"]).sum() + (mus * g["v_mus"]).sum(), cov)[0]
    torch.testing.assert_close(grad, g["grad"], atol=1e-9, rtol=1e-9)


@pytest.mark.parametrize("case", range(2))
def test_conics_nonpositive_det3(golden, case):
    g = golden["conics_nonpositive"][case]
    conics, mus = O.conics_mu(g["covars"], 0.0)
    torch.testing.assert_close(conics, g["conics"], atol=1e-12, rtol=1e-9)
    assert (mus == 0).all()


def test_degenerate_2d_covariance_gives_zeros():
    cov = torch.tensor([[[1e-6, 0.0, 0.0, 1e-6, 0.0, 1.0]]], dtype=torch.float64)
    conics, mus = O.conics_mu(cov, 1e-8)
    assert (conics == 0).all() and (mus == 0).all()


def test_raster_matches_golden(golden):
    g = golden["raster"]
    m = g["means2d"].clone().requires_grad_(True)
    c = g["conics"].clone().requires_grad_(True)
    o = g["opacity"].clone().requires_grad_(True)
    mu = g["mus"].clone().requires_grad_(True)
    mask = torch.ones((1, 2, 16, 16), dtype=torch.bool)
    img = O.rasterize(m, c, o, mu, mask, 16, 16)
    torch.testing.assert_close(img.detach(), g["image"], atol=1e-6, rtol=1e-5)
    grads = torch.autograd.grad((img * g["weight"]).sum(), (m, c, o, mu))
    for a, k in zip(grads, ("v_means2d", "v_conics", "v_opacity", "v_mus")):
        torch.testing.assert_close(a, g[k], atol=1e-5, rtol=1e-5)


def test_voxel_matches_golden(golden):
    g = golden["voxel"]
    m = g["means3d"].clone().requires_grad_(True)
    c = g["conics"].clone().requires_grad_(True)
    o = g["opacity"].clone().requires_grad_(True)
    rects = np.array([[0, 1, 0, 1, 0, 1]] * 2)
    valid = np.array([True, True])
    vol = O.voxelize(m, c, o, rects, valid, 8, 8, 8, 8)
    torch.testing.assert_close(vol.detach(), g["volume"], atol=1e-6, rtol=1e-5)
    grads = torch.autograd.grad((vol * g["weight"]).sum(), (m, c, o))
    for a, k in zip(grads, ("v_means3d", "v_conics", "v_opacity")):
        torch.testing.assert_close(a, g[k], atol=1e-5, rtol=1e-5)


def test_tile_rects_near_integer_boundaries():
    """Adversarial cases of the tile bound arithmetic (IsectTilesKernel.cu:92-103):
    bounds that land exactly on tile edges, radii crossing the image border,
    non-finite means and zero radii."""
    means = np.array([[[32.0, 32.0], [31.999998, 16.0], [-5.0, 8.0], [np.nan, 3.0],
                       [200.0, 8.0], [8.0, 8.0]]], dtype=np.float32)
    radii = np.array([[[16, 16], [1, 1], [6, 2], [3, 3], [100, 4], [0, 5]]], dtype=np.int32)
    rects, valid, counts = O.tile_rects_2d(means, radii, 16, 4, 4)
    # [16, 48) -> tiles [1, 3)
    assert tuple(rects[0, 0]) == (1, 3, 1, 3) and counts[0, 0] == 4
    # x in [30.999998, 32.999998): floor(1.9375) = 1, ceil(2.0624999) = 3
    assert tuple(rects[0, 1][:2]) == (1, 3)
    # left of the image: [-11, 1) -> tiles [0, 1)
    assert tuple(rects[0, 2][:2]) == (0, 1) and valid[0, 2]
    assert not valid[0, 3] and counts[0, 3] == 0
    # [100, 300) clamped to the 4-tile grid -> [6, 4) empty
    assert not valid[0, 4]
    assert not valid[0, 5]


def test_binning_is_stable_and_offsets_encode_runs():
    rng = np.random.default_rng(0)
    C, N, ntx, nty = 3, 40, 5, 4
    means = rng.uniform(-10, 90, size=(C, N, 2)).astype(np.float32)
    radii = rng.integers(0, 25, size=(C, N, 2)).astype(np.int32)
    rects, valid, counts = O.tile_rects_2d(means, radii, 16, ntx, nty)
    keys, vals, offs = O.bin_2d(rects, valid, ntx, nty)
    k2, v2, o2 = O.bin_2d_fast(rects, valid, ntx, nty)
    assert (keys == k2).all() and (vals == v2).all() and (offs == o2).all()
    assert keys.size == counts.sum()
    assert (np.diff(keys) >= 0).all()
    same = np.diff(keys) == 0
    assert (np.diff(vals)[same] > 0).all(), "equal keys must keep ascending flattened ids"
    flat = offs.reshape(-1)
    for k in range(C * ntx * nty):
        lo = flat[k]
        hi = flat[k + 1] if k + 1 < flat.size else keys.size
        assert (keys[lo:hi] == k).all()
        assert lo == np.searchsorted(keys, k)


def test_offsets_of_empty_key_array_are_zero():
    assert (O.offsets_from_keys(np.zeros(0, np.int64), 7) == 0).all()


def test_bin_3d_order_and_counts():
    rng = np.random.default_rng(1)
    N, nt = 50, 4
    m = rng.uniform(-4, 36, size=(N, 3)).astype(np.float32)
    r = rng.integers(0, 9, size=(N, 3)).astype(np.int32)
    rects, valid, counts = O.brick_rects_3d(m, r, 8, nt, nt, nt)
    keys, vals, offs = O.bin_3d(rects, valid, nt, nt, nt)
    assert keys.size == counts.sum()
    same = np.diff(keys) == 0
    assert (np.diff(vals)[same] > 0).all()
    assert offs.shape == (nt, nt, nt)


def test_saturating_brick_bounds():
    """Negative bounds saturate to 0 and large ones clamp to the grid
    (IsectTiles3DKernel.cu:93-98)."""
    m = np.array([[-30.0, 4.0, 4.0], [4.0, 4.0, 400.0]], dtype=np.float32)
    r = np.array([[5, 2, 2], [2, 2, 500]], dtype=np.int32)
    rects, valid, counts = O.brick_rects_3d(m, r, 8, 4, 4, 4)
    assert not valid[0]  # x range [0, 0)
    assert tuple(rects[1][4:]) == (0, 4) and valid[1]


def test_projection_pipeline_small_case_consistent():
    """The oracle's own projection pipeline: image equals a dense evaluation
    restricted to the binned tiles, radii are non-negative."""
    import r2s_workloads as wl

    cfg = wl.CONFIGS[0]
    m, q, s, o = wl.make_gaussians(cfg, n=64)
    vm, K = wl.make_cameras(2, 32, total=2)
    img, m2, radii, (rects, valid, counts) = O.projection_forward(
        m, q, s, o, vm, K, width=32, height=32, tile=16, eps2d=1e-8, clip=3.0,
        smin=wl.SCALE_MIN, smax=wl.SCALE_MAX)
    assert img.shape == (2, 32, 32) and torch.isfinite(img).all()
    assert (radii >= 0).all()
    assert counts.sum() > 0


def test_rel_l2_helper():
    a = torch.tensor([1.0, 2.0])
    assert rel_l2(a, a) == 0.0
    assert math.isclose(O.rel_l2(torch.tensor([1.0, 0.0]), torch.tensor([1.0, 1.0])), 1 / math.sqrt(2))
