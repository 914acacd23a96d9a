"""The forward's culling table (cull_ranges of r2s_raster_splats_fwd_f32):
writing it leaves the image bit for bit unchanged, and the backward that
reads it agrees with the backward that recomputes the ranges to float
rounding, on full and ragged detectors."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("W,H", [(128, 128), (117, 90)])
def test_cull_table_roundtrip(W, H):
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as Wr

    m, q, s, o = (t.cuda() for t in wl.make_gaussians(wl.CONFIGS[1], n=20000, seed=6))
    vm, K = (t.cuda() for t in wl.make_cameras(3, 128))
    cov, _, op = Wr.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
    ntx, nty = (W + 15) // 16, (H + 15) // 16
    _, _, splats, rects, _ = Wr.fused_project(m, cov, op, vm, K, W, H, 16, ntx, nty, wl.EPS2D,
                                              wl.RADIUS_CLIP)
    offs, fids, _ = Wr.fused_bin(rects, 3, m.size(0), ntx * nty, ntx, 0)
    offs = offs.view(3, nty, ntx)
    cull = torch.full(fids.shape, -1, dtype=torch.int16, device="cuda")
    img_t = Wr.fused_raster_fwd(splats, offs, fids, 3, m.size(0), W, H, 16, ntx, nty, cull=cull)
    img = Wr.fused_raster_fwd(splats, offs, fids, 3, m.size(0), W, H, 16, ntx, nty)
    assert torch.equal(img, img_t) and img.abs().max() > 0
    # every entry written: 4-bit ranges, empty ones as (1, 0)
    v = cull.to(torch.int32) & 0xFFFF
    c_lo, c_hi, r_lo, r_hi = v & 15, (v >> 4) & 15, (v >> 8) & 15, v >> 12
    live = (c_lo <= c_hi) & (r_lo <= r_hi)
    assert bool((live | ((c_lo == 1) & (c_hi == 0)) | ((r_lo == 1) & (r_hi == 0))).all())
    assert live.float().mean() > 0.5
    g = torch.Generator(device="cuda").manual_seed(1)
    v_img = torch.randn(img.shape, generator=g, device="cuda")
    for absgrad in (True, False):
        st_t = Wr.fused_raster_bwd(splats, offs, fids, v_img, 3, m.size(0), W, H, 16, ntx, nty,
                                   absgrad, cull=cull)
        st = Wr.fused_raster_bwd(splats, offs, fids, v_img, 3, m.size(0), W, H, 16, ntx, nty,
                                 absgrad)
        rel = ((st_t.double() - st.double()).norm() / st.double().norm()).item()
        assert rel < 1e-6, (absgrad, rel)
