"""Model adapter (r2s_model.GaussianAdapter) checks that need no GPU: the
reference's option validation and errors (src/models/gaussian_model.py:
280-492) and the rigid inverse of the camera poses (src/utils/math.py:5-32)."""
import math

import pytest
import torch

import r2s_model as M
import r2s_workloads as wl


def _adapter(**kw):
    m, q, s, o = wl.make_gaussians(wl.CONFIGS[0], n=16)
    return M.GaussianAdapter(m, q, s, o, **kw)


def test_invert_rigid_transform_matches_the_matrix_inverse():
    c2w = torch.stack([wl.camtoworld(2 * math.pi * k / 7) for k in range(7)])
    inv = M.invert_rigid_transform(c2w)
    torch.testing.assert_close(inv, torch.linalg.inv(c2w), rtol=1e-12, atol=1e-12)
    assert inv.is_contiguous() and inv.dtype == torch.float64
    with pytest.raises(ValueError, match=r"Expected transform shape \[..., 4, 4\]"):
        M.invert_rigid_transform(torch.eye(3))


@pytest.mark.parametrize("kw,err,msg", [
    (dict(packed=True), ValueError, "packed=True"),
    (dict(sparse_grad=True), ValueError, "sparse_grad=True"),
    (dict(rasterize_mode="antialiased"), ValueError, "rasterize_mode='classic'"),
    (dict(camera_model="ortho"), ValueError, "camera_model='pinhole'"),
    (dict(backgrounds=None), TypeError, "Unsupported rasterization options"),
    (dict(viewmats=torch.eye(4)[None].expand(3, 4, 4)), ValueError, "same shape as camtoworlds"),
])
def test_rasterize_rejects_unsupported_options(kw, err, msg):
    a = _adapter()
    c2w = torch.eye(4)[None].expand(2, 4, 4).contiguous()
    with pytest.raises(err, match=msg):
        a.rasterize(c2w, torch.eye(3)[None].expand(2, 3, 3), 64, 64, **kw)


def test_prepare_requires_scalar_sigmoid_bounds():
    with pytest.raises(RuntimeError, match="bounded sigmoid scales"):
        _adapter(scale_min=None, scale_max=None).prepare_gaussians()
    with pytest.raises(RuntimeError, match="scalar scale bounds"):
        _adapter(scale_min=[1e-4, 1e-4, 1e-4], scale_max=[1.0, 1.0, 1.0]).prepare_gaussians()


def test_voxelize_and_backward_argument_errors():
    a = _adapter()
    assert a.voxelize((8, 8, 8), None) is None
    with pytest.raises(TypeError, match="Unsupported voxelization options"):
        a.voxelize((8, 8, 8), torch.tensor([[-0.5] * 3, [0.5] * 3]), foo=1)
    with pytest.raises(TypeError, match="requires an ExplicitGaussianState"):
        a.backward_explicit(object())
