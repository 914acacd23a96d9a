"""Edge cases of the float32 op layer (the fused kernels) against the live
reference build: ragged detector tiles and voxel bricks, Gaussians that are
all culled, non-finite means, a single Gaussian, very large footprints."""

import pytest
import torch

from _helpers import REL_L2_F32, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    from oracle.ref_harness import ReferencePipeline

    return ReferencePipeline()


def _run_both(ref, m, q, s, o, vm, K, W, H, G, ranges=None, centers=None):
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    ranges = torch.ones(3, device="cuda") if ranges is None else ranges
    centers = torch.zeros(3, device="cuda") if centers is None else centers
    params = [t.clone().requires_grad_(True) for t in (m, q, s, o)]
    st = E.prepare_explicit_gaussians(params[1], params[2], params[3], scale_min=wl.SCALE_MIN,
                                      scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(st, params[0], vm, K, img_w=W, img_h=H, tile_size=16,
                               eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP, absgrad=True)
    vox = E.explicit_voxelize(st, params[0], ranges, centers, dim2=G, dim1=G + 3, dim0=G + 5,
                              tile_size=8, eps3d=wl.EPS3D, radius_clip=wl.RADIUS_CLIP)
    g = torch.Generator(device="cuda").manual_seed(3)
    v_img = torch.randn(res.image.shape, generator=g, device="cuda")
    v_vol = torch.randn(vox.volume.shape, generator=g, device="cuda")
    (res.image * v_img).sum().backward()
    (vox.volume * v_vol).sum().backward()
    E.explicit_backward(st, *params)
    cov, ms, op = ref.prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
    p = ref.rasterize_forward(m, cov, op, vm, K, W, H, 16, wl.EPS2D, wl.RADIUS_CLIP)
    v = ref.voxelize_forward(m, cov, ms, op, ranges, centers, G, G + 3, G + 5, 8, wl.EPS3D,
                             wl.RADIUS_CLIP)
    theirs = ref.explicit_backward(p, v_img, v, v_vol, m, q, s, o, cov, op, wl.SCALE_MIN,
                                   wl.SCALE_MAX, absgrad=True)
    return st, res, vox, params, p, v, theirs


def _check(st, res, vox, params, p, v, theirs, grads=True):
    assert torch.equal(res.radii, p["radii"])
    assert torch.equal(st.projection.buffers.tile_offsets, p["tile_offsets"])
    assert torch.equal(st.projection.buffers.flatten_ids, p["flatten_ids"])
    assert torch.equal(vox.radii, v["radii"])
    assert torch.equal(st.voxel.buffers.tile_offsets, v["tile_offsets"])
    assert torch.equal(st.voxel.buffers.flatten_ids, v["flatten_ids"])
    for a, b in ((res.image, p["output"]), (vox.volume, v["output"])):
        assert torch.isfinite(a).all()
        if b.abs().max() > 0:
            assert rel_l2(a, b) < REL_L2_F32
        else:
            assert (a == 0).all()
    if grads:
        for k, t in zip(("means", "quats", "scales", "opacities"), params):
            ref_g = theirs[k]
            if ref_g.abs().max() == 0:
                assert (t.grad == 0).all(), k
            else:
                assert rel_l2(t.grad, ref_g) < REL_L2_F32, (k, rel_l2(t.grad, ref_g))


def _workload(n, seed, views=3, det=100):
    import r2s_workloads as wl

    m, q, s, o = (t.cuda() for t in wl.make_gaussians(wl.CONFIGS[0], n=n, seed=seed))
    vm, K = wl.make_cameras(views, det, total=7)
    return m, q, s, o, vm.cuda(), K.cuda()


def test_ragged_tiles_and_bricks(ref):
    m, q, s, o, vm, K = _workload(600, 11, det=100)
    # detector 100 x 70 (tiles 7 x 5, ragged), grid 21 x 24 x 26 (ragged bricks)
    out = _run_both(ref, m, q, s, o, vm, K, 100, 70, 21)
    _check(*out)


def test_all_gaussians_culled(ref):
    m, q, s, o, vm, K = _workload(64, 12)
    m = m + torch.tensor([0.0, 0.0, 50.0], device="cuda")  # far outside view and grid
    out = _run_both(ref, m, q, s, o, vm, K, 100, 100, 16)
    st, res, vox, params, p, v, theirs = out
    assert st.projection.buffers.flatten_ids.numel() == p["flatten_ids"].numel()
    assert (res.image == 0).all() and (vox.volume == 0).all()
    _check(*out)


def test_non_finite_means_are_culled_like_the_reference(ref):
    m, q, s, o, vm, K = _workload(200, 13)
    m[0] = float("nan")
    m[1, 2] = float("inf")
    m[2, 0] = -float("inf")
    out = _run_both(ref, m, q, s, o, vm, K, 96, 96, 16)
    _check(*out, grads=False)
    st, res, vox, params, p, v, theirs = out
    for k, t in zip(("means", "quats", "scales", "opacities"), params):
        keep = torch.ones(t.shape[0], dtype=torch.bool, device="cuda")
        keep[:3] = False
        assert rel_l2(t.grad[keep], theirs[k][keep]) < REL_L2_F32, k


def test_single_gaussian(ref):
    m, q, s, o, vm, K = _workload(1, 14, views=1)
    m.zero_()
    out = _run_both(ref, m, q, s, o, vm, K, 64, 64, 16)
    _check(*out)


def test_large_footprints(ref):
    import r2s_workloads as wl

    m, q, s, o, vm, K = _workload(40, 15)
    # wide anisotropic Gaussians covering many tiles and bricks (an isotropic
    # covariance would make the quaternion gradient vanish)
    g = torch.Generator().manual_seed(15)
    wide = torch.tensor([0.4, 0.25, 0.15]) * (0.8 + 0.4 * torch.rand(40, 3, generator=g))
    s = wl.inverse_scale(wide).float().cuda()
    out = _run_both(ref, m, q, s, o, vm, K, 128, 128, 24)
    _check(*out)


def test_view_batches_beyond_the_record_limit(monkeypatch):
    """When the intersection records of all views pass the int32 limit of one
    binning, the float32 path bins and rasterizes in view batches; forced here
    with a small limit, the image and gradients equal the single-batch run."""
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W
    from r2splat.ops import explicit as E

    cfg = wl.CONFIGS[1]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg, n=20000))
    vm, K = wl.make_cameras(6, 128, total=6)
    vm, K = vm.cuda(), K.cuda()
    g = torch.Generator(device="cuda").manual_seed(4)
    v_img = torch.randn((6, 128, 128), generator=g, device="cuda")

    def run():
        params = [t.clone().requires_grad_(True) for t in (m, q, s, o)]
        st = E.prepare_explicit_gaussians(params[1], params[2], params[3],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        res = E.explicit_rasterize(st, params[0], vm, K, img_w=128, img_h=128, tile_size=16,
                                   eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP, absgrad=True)
        (res.image * v_img).sum().backward()
        E.explicit_backward(st, *params)
        return st, res, params

    st1, res1, p1 = run()
    n = st1.projection.buffers.flatten_ids.numel()
    monkeypatch.setattr(W, "MAX_RECORDS_PER_BATCH", n // 4)
    st2, res2, p2 = run()
    batches = st2.projection.buffers.view_batches
    assert batches is not None and len(batches) >= 4
    assert sum(ids.numel() for _, _, ids in batches) == n
    assert torch.equal(res2.image, res1.image)
    for a, b in zip(p2, p1):
        assert rel_l2(a.grad, b.grad) < 1e-6
    assert rel_l2(res2.means2d.absgrad, res1.means2d.absgrad) < 1e-6
