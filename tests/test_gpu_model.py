"""Model adapter (r2s_model.GaussianAdapter) on the GPU: the reference's
GaussianModel.rasterize / voxelize / backward_explicit layouts and info dict
(src/models/gaussian_model.py:319-492) over the ops of this package."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _scene():
    import r2s_workloads as wl

    m, q, s, o = (t.cuda() for t in wl.make_gaussians(wl.CONFIGS[0], n=2000, seed=9))
    c2w = torch.stack([wl.camtoworld(2 * math.pi * k / 3) for k in range(3)]).float().cuda()
    K = wl.make_cameras(3, 96)[1].cuda()
    bbox = torch.tensor([[-0.5, -0.5, -0.5], [0.5, 0.5, 0.5]], device="cuda")
    return m, q, s, o, c2w, K, bbox


def test_inference_render_and_volume_layouts():
    import r2s_model as M
    import r2s_workloads as wl
    from r2splat.ops import inference_rasterize, inference_voxelize, prepare_inference_gaussians

    m, q, s, o, c2w, K, bbox = _scene()
    a = M.GaussianAdapter(m, q, s, o)
    renders, info = a.rasterize(c2w, K, 96, 80)
    st = prepare_inference_gaussians(q, s, o, scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
    vm = M.invert_rigid_transform(c2w)
    res = inference_rasterize(st, m, vm, K, img_w=96, img_h=80, tile_size=16, eps2d=wl.EPS2D,
                              radius_clip=wl.RADIUS_CLIP)
    assert renders.shape == (3, 96, 80, 1)
    assert torch.equal(renders[..., 0], res.image.transpose(1, 2))
    assert torch.equal(info["radii"], res.radii.amax(-1))
    assert torch.equal(info["means2d"], res.means2d)
    assert info["gaussian_ids"].shape == (3, 2000)
    assert torch.equal(info["gaussian_ids"][2], torch.arange(2000, device="cuda"))
    assert (info["width"], info["height"], info["n_cameras"]) == (96, 80, 3)
    vol = a.voxelize((24, 20, 16), bbox)
    ref = inference_voxelize(st, m, bbox[1] - bbox[0], (bbox[0] + bbox[1]) / 2, dim2=24, dim1=20,
                             dim0=16, tile_size=8, eps3d=wl.EPS3D, radius_clip=wl.RADIUS_CLIP)
    assert vol.shape == (16, 20, 24, 1) and torch.equal(vol[..., 0], ref.volume)


def test_explicit_training_step_through_the_adapter():
    """prepare(explicit) -> rasterize + voxelize -> loss backward ->
    backward_explicit gives the gradients of the same step on the ops."""
    import r2s_model as M
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    m, q, s, o, c2w, K, bbox = _scene()
    g = torch.Generator(device="cuda").manual_seed(3)
    w_img = torch.randn(3, 96, 96, 1, generator=g, device="cuda")
    w_vol = torch.randn(16, 16, 16, 1, generator=g, device="cuda")

    pa = [torch.nn.Parameter(t.clone()) for t in (m, q, s, o)]
    a = M.GaussianAdapter(*pa)
    st = a.prepare_gaussians(explicit=True)
    renders, info = a.rasterize(c2w, K, 96, 96, absgrad=True, gaussian_state=st)
    vol = a.voxelize((16, 16, 16), bbox, gaussian_state=st)
    ((renders * w_img).sum() + (vol * w_vol).sum()).backward()
    a.backward_explicit(st)

    pb = [torch.nn.Parameter(t.clone()) for t in (m, q, s, o)]
    st2 = E.prepare_explicit_gaussians(pb[1], pb[2], pb[3], scale_min=wl.SCALE_MIN,
                                       scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(st2, pb[0], M.invert_rigid_transform(c2w), K, img_w=96, img_h=96,
                               tile_size=16, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                               absgrad=True)
    vres = E.explicit_voxelize(st2, pb[0], bbox[1] - bbox[0], (bbox[0] + bbox[1]) / 2, dim2=16,
                               dim1=16, dim0=16, tile_size=8, eps3d=wl.EPS3D,
                               radius_clip=wl.RADIUS_CLIP)
    ((res.image * w_img[..., 0].transpose(1, 2)).sum() + (vres.volume * w_vol[..., 0]).sum()).backward()
    E.explicit_backward(st2, *pb)
    for x, y in zip(pa, pb):
        torch.testing.assert_close(x.grad, y.grad, rtol=1e-4, atol=1e-6)
    assert info["means2d"].absgrad is not None
    with pytest.raises(RuntimeError, match="only run once"):
        a.backward_explicit(st)
