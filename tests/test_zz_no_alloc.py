"""The rasterizer backward that allocates nothing, against the allocating one.

r2s_rasterize_to_pixels_bwd_noalloc_f32 serves host programs that cannot
give the library scratch memory (their device memory belongs to an allocator
the plugin may not call, and their binding passes only inputs and outputs).
It keeps its scratch in a static device array of the library.  This test
calls it through the C ABI twice in a row -- the second call must not see
the first call's statistics, which stay in the shared array -- and compares
every output with r2s_rasterize_to_pixels_bwd (caller scratch) on the same
inputs, within the float32 tolerance of the other parity tests.  It also
checks that a call beyond the array's stated limit is rejected.
"""
import ctypes

import pytest
import torch

from _helpers import REL_L2_F32, rel_l2

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _raster_inputs():
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W

    cfg = wl.CONFIGS[0]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg, n=2048))
    vm, K = wl.make_cameras(3, 128, total=3)
    vm, K = vm.cuda(), K.cuda()
    covars, _ = W.parameter_transform_fwd(q, s, wl.SCALE_MIN, wl.SCALE_MAX)
    means2d, cov2d, radii = W.world_to_image_projection_fwd(m, covars, vm, K, 128, 128, wl.EPS2D,
                                                            wl.RADIUS_CLIP)
    conics, mus = W.conics_mu_fwd(cov2d, wl.EPS2D)
    opacity = torch.nn.functional.softplus(o)[None].expand(3, -1).contiguous()
    _, isect_ids, flatten_ids = W.isect_tiles(means2d, radii, 16, 8, 8)
    offsets = W.isect_offset_encode(isect_ids, 3, 8, 8)
    return dict(means2d=means2d, conics=conics, opacity=opacity, mus=mus, offsets=offsets,
                isect_ids=isect_ids, flatten_ids=flatten_ids, C=3, N=2048, W=128, H=128)


def _noalloc_call(lib, d, v_img, mode):
    C, N = d["C"], d["N"]
    outs = dict(abs=torch.full((C, N, 2), float("nan"), device="cuda"),
                m2=torch.full((C, N, 2), float("nan"), device="cuda"),
                con=torch.full((C, N, 3), float("nan"), device="cuda"),
                op=torch.full((C, N), float("nan"), device="cuda"),
                mu=torch.full((C, N), float("nan"), device="cuda"))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.r2s_rasterize_to_pixels_bwd_noalloc_f32(
        mode, _ptr(d["means2d"]), _ptr(d["conics"]), _ptr(d["opacity"]), _ptr(d["mus"]),
        _ptr(d["offsets"]), _ptr(d["flatten_ids"]), _ptr(v_img), C, N, d["flatten_ids"].numel(),
        d["W"], d["H"], 16, 8, 8, _ptr(outs["abs"]), _ptr(outs["m2"]), _ptr(outs["con"]),
        _ptr(outs["op"]), _ptr(outs["mu"]), stream)
    return rc, outs


def test_noalloc_backward_matches_allocating_backward_on_two_calls():
    from r2splat.cuda import _wrapper as W
    from r2splat.cuda._backend import _C

    d = _raster_inputs()
    assert d["flatten_ids"].numel() > 0
    for call, mode in enumerate((1, 0)):
        g = torch.Generator(device="cuda").manual_seed(11 + call)
        v_img = torch.randn((d["C"], d["H"], d["W"]), generator=g, device="cuda")
        rc, outs = _noalloc_call(_C, d, v_img, mode)
        assert rc == 0, W._last_error()
        if mode == 1:
            ref = W.rasterize_to_pixels_bwd_per_gaussian(
                d["means2d"], d["conics"], d["opacity"], d["mus"], d["offsets"], d["isect_ids"],
                d["flatten_ids"], v_img, d["W"], d["H"], 16, True)
        else:
            ref = W.rasterize_to_pixels_bwd(
                d["means2d"], d["conics"], d["opacity"], d["mus"], d["offsets"], d["flatten_ids"],
                v_img, d["W"], d["H"], 16, True)
        torch.cuda.synchronize()
        for key, expected in zip(("abs", "m2", "con", "op", "mu"), ref):
            assert torch.isfinite(outs[key]).all(), f"call {call}: {key} not fully written"
            err = rel_l2(outs[key], expected)
            assert err <= REL_L2_F32, f"call {call}: {key} rel-L2 {err:.3e}"


def test_noalloc_backward_rejects_sizes_beyond_its_scratch():
    from r2splat.cuda import _wrapper as W
    from r2splat.cuda._backend import _C

    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _C.r2s_rasterize_to_pixels_bwd_noalloc_f32(1, None, None, None, None, None, None, None,
                                                    4, 40000, 1, 64, 64, 16, 4, 4, None, None,
                                                    None, None, None, stream)
    assert rc == 4  # R2S_ERR_UNSUPPORTED
    assert "static scratch" in W._last_error()
    # sizes whose product overflows int64 are rejected too, not wrapped
    rc = _C.r2s_rasterize_to_pixels_bwd_noalloc_f32(1, None, None, None, None, None, None, None,
                                                    2 ** 40, 2 ** 40, 1, 64, 64, 16, 4, 4, None,
                                                    None, None, None, None, stream)
    assert rc == 4
    assert "static scratch" in W._last_error()
