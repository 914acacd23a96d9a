"""Known-answer tests of the 18 low-level operators on the GPU.

Ports of the reference's CUDA operator tests
(tests/test_cuda_gaussian_ops.py:53-380): the answers are the dense PyTorch
references of that suite, evaluated by tests/golden/make_golden.py into
tests/golden/kat.pt.  Tolerances: the reference suite's atol = rtol = 3e-4
for float32 (1e-9 for float64), and additionally the rel-L2 <= 1e-5 bar of
this project where the golden is exact.
"""
import pytest
import torch

from _helpers import REL_L2_F32, cuda, load_golden, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden():
    return load_golden()


@pytest.fixture(scope="module")
def W():
    from r2splat.cuda import _wrapper

    assert _wrapper.is_cuda_extension_available(), "libr2s.so did not load on a CUDA machine"
    return _wrapper


def test_extension_is_loaded(W):
    from r2splat.cuda._backend import library_path
    import os

    assert os.path.exists(library_path())


def test_parameter_transform_matches_dense_reference(W, golden):
    g = golden["param"]
    covars, max_scales = W.parameter_transform_fwd(cuda(g["quats"]), cuda(g["raw_scales"]),
                                                   g["scale_min"], g["scale_max"])
    torch.testing.assert_close(covars.cpu(), g["covars"], atol=3e-4, rtol=3e-4)
    torch.testing.assert_close(max_scales.cpu(), g["max_scales"], atol=3e-4, rtol=3e-4)
    assert rel_l2(covars, g["covars"]) < REL_L2_F32
    v_q, v_s = W.parameter_transform_bwd(cuda(g["quats"]), cuda(g["raw_scales"]), g["scale_min"],
                                         g["scale_max"], cuda(g["v_covars"]))
    torch.testing.assert_close(v_q.cpu(), g["v_quats"], atol=3e-4, rtol=3e-4)
    torch.testing.assert_close(v_s.cpu(), g["v_raw_scales"], atol=3e-4, rtol=3e-4)
    assert rel_l2(v_q, g["v_quats"]) < 1e-5
    assert rel_l2(v_s, g["v_raw_scales"]) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("case", range(4))
def test_conics_mu_near_det3_threshold(W, golden, dtype, case):
    """Reference kernel semantics (csrc/ConicsMuBwd.cu:126-161): the mu term
    of the gradient is applied only when the blurred det3 exceeds 1e-9; the
    reference suite's test of the same inputs expects it for every positive
    det3, which the reference kernel does not do.  This build matches the
    kernel: full gradient above the cut-off, conic-only gradient below."""
    g = golden["conics_mu"][case]
    tol = 3e-4 if dtype == torch.float32 else 1e-9
    cov = cuda(g["covars"], dtype)
    conics, mus = W.conics_mu_fwd(cov, g["eps"])
    torch.testing.assert_close(conics.cpu(), g["conics"].to(dtype), atol=tol, rtol=tol)
    torch.testing.assert_close(mus.cpu(), g["mus"].to(dtype), atol=tol, rtol=tol)
    assert (mus > 0).all()
    grad = W.conics_mu_bwd(cov, g["eps"], conics, mus, cuda(g["v_conics"], dtype),
                           cuda(g["v_mus"], dtype))
    above = (g["det3"] > 1e-9)[..., None]
    expected = torch.where(above, g["grad"], g["grad_conic_only"]).to(dtype)
    torch.testing.assert_close(grad.cpu(), expected, atol=tol, rtol=tol)
    assert (grad[..., 5].cpu()[above[..., 0]] > 0).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("case", range(2))
def test_conics_mu_nonpositive_det3_keeps_conic_gradients(W, golden, dtype, case):
    g = golden["conics_nonpositive"][case]
    tol = 3e-4 if dtype == torch.float32 else 1e-9
    cov = cuda(g["covars"], dtype)
    conics, mus = W.conics_mu_fwd(cov, 0.0)
    grad = W.conics_mu_bwd(cov, 0.0, conics, mus, torch.ones_like(conics), torch.ones_like(mus))
    torch.testing.assert_close(conics.cpu(), g["conics"].to(dtype), atol=tol, rtol=tol)
    torch.testing.assert_close(mus.cpu(), torch.zeros_like(mus.cpu()))
    torch.testing.assert_close(grad.cpu(), g["grad"].to(dtype), atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_conics_mu_rejects_degenerate_2d_covariance(W, dtype):
    cov = torch.tensor([[[1e-6, 0.0, 0.0, 1e-6, 0.0, 1.0]]], dtype=dtype, device="cuda")
    conics, mus = W.conics_mu_fwd(cov, 1e-8)
    grad = W.conics_mu_bwd(cov, 1e-8, conics, mus, torch.ones_like(conics), torch.ones_like(mus))
    assert (conics == 0).all() and (mus == 0).all() and (grad == 0).all()


@pytest.mark.parametrize("primitive_backward", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_raster_forward_backward_matches_dense_reference(W, golden, primitive_backward, dtype):
    g = golden["raster"]
    m, c, o, mu = (cuda(g[k], dtype) for k in ("means2d", "conics", "opacity", "mus"))
    offsets = torch.zeros((1, 1, 1), dtype=torch.int32, device="cuda")
    flatten_ids = torch.arange(2, dtype=torch.int32, device="cuda")
    isect_ids = torch.zeros(2, dtype=torch.int64, device="cuda")
    img = W.rasterize_to_pixels_fwd(m, c, o, mu, offsets, flatten_ids, 16, 16, 16)
    torch.testing.assert_close(img.cpu(), g["image"].to(dtype), atol=3e-4, rtol=3e-4)
    assert rel_l2(img, g["image"]) < 1e-5
    weight = cuda(g["weight"], dtype)
    if primitive_backward:
        grads = W.rasterize_to_pixels_bwd_per_gaussian(m, c, o, mu, offsets, isect_ids, flatten_ids,
                                                       weight, 16, 16, 16, True)
    else:
        grads = W.rasterize_to_pixels_bwd(m, c, o, mu, offsets, flatten_ids, weight, 16, 16, 16,
                                          True)
    for actual, key in zip(grads[1:], ("v_means2d", "v_conics", "v_opacity", "v_mus")):
        torch.testing.assert_close(actual.cpu(), g[key].to(dtype), atol=3e-4, rtol=3e-4)
        assert rel_l2(actual, g[key]) < 2e-5
    assert grads[0].shape == m.shape and torch.isfinite(grads[0]).all()


@pytest.mark.parametrize("primitive_backward", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_voxel_forward_backward_matches_dense_reference(W, golden, primitive_backward, dtype):
    g = golden["voxel"]
    m, c, o = (cuda(g[k], dtype) for k in ("means3d", "conics", "opacity"))
    offsets = torch.zeros((1, 1, 1), dtype=torch.int32, device="cuda")
    flatten_ids = torch.arange(2, dtype=torch.int32, device="cuda")
    isect_ids = torch.zeros(2, dtype=torch.int64, device="cuda")
    vol = W.voxelize_to_voxels_fwd(m, c, o, offsets, flatten_ids, 8, 8, 8, 8)
    torch.testing.assert_close(vol.cpu(), g["volume"].to(dtype), atol=3e-4, rtol=3e-4)
    assert rel_l2(vol, g["volume"]) < 1e-5
    weight = cuda(g["weight"], dtype)
    if primitive_backward:
        grads = W.voxelize_to_voxels_bwd_per_gaussian(m, c, o, offsets, isect_ids, flatten_ids,
                                                      weight, 8, 8, 8, 8)
    else:
        grads = W.voxelize_to_voxels_bwd(m, c, o, offsets, flatten_ids, weight, 8, 8, 8, 8)
    for actual, key in zip(grads, ("v_means3d", "v_conics", "v_opacity")):
        torch.testing.assert_close(actual.cpu(), g[key].to(dtype), atol=3e-4, rtol=3e-4)
        assert rel_l2(actual, g[key]) < 2e-5


def test_empty_inputs_return_zero_or_empty(W):
    dev = "cuda"
    m = torch.zeros((1, 0, 2), device=dev)
    c = torch.zeros((1, 0, 3), device=dev)
    o = torch.zeros((1, 0), device=dev)
    offsets = torch.zeros((1, 2, 2), dtype=torch.int32, device=dev)
    fl = torch.zeros((0,), dtype=torch.int32, device=dev)
    img = W.rasterize_to_pixels_fwd(m, c, o, o, offsets, fl, 32, 32, 16)
    assert img.shape == (1, 32, 32) and (img == 0).all()
    tpg, ids, fids = W.isect_tiles(m, torch.zeros((1, 0, 2), dtype=torch.int32, device=dev), 16, 2, 2)
    assert tpg.shape == (1, 0) and ids.numel() == 0 and fids.numel() == 0
    off = W.isect_offset_encode(ids, 1, 2, 2)
    assert off.shape == (1, 2, 2) and (off == 0).all()
