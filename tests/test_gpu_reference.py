"""Parity against the live reference build (oracle/_ref, the reference's own
CUDA sources compiled for sm_100a by oracle/build_ref.py).

Integer outputs (radii, tiles per Gaussian, sorted keys, flatten ids, tile
offsets) must be identical; floating-point outputs within rel-L2 1e-5
(float32).  Inputs are seeded synthetic workloads with the shapes of
benchmark configs 0, 1 and 2: config 1 reduced to 8 views; config 2 both at
4 views and at its full size (500k Gaussians, all 75 views of the orbit,
512^2 detector, 256^3 grid), so every view the benchmark bins is compared.
"""
import os

import pytest
import torch

from _helpers import REL_L2_F32, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    from oracle.ref_harness import ReferencePipeline, REF_SO

    assert os.path.exists(REF_SO), "reference build missing: run python oracle/build_ref.py"
    return ReferencePipeline()


@pytest.fixture(scope="module")
def W():
    from r2splat.cuda import _wrapper

    return _wrapper


def _workload(cfg_id, n=None, views=None, det=None, grid=None):
    import r2s_workloads as wl

    cfg = wl.CONFIGS[cfg_id]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg, n=n))
    views = cfg.n_views if views is None else views
    det = cfg.detector if det is None else det
    grid = cfg.grid if grid is None else grid
    vm, K = wl.make_cameras(views, det, total=cfg.n_views)
    rng, ctr = wl.unit_cube_box()
    return dict(means=m, quats=q, scales=s, opac=o, viewmats=vm.cuda(), Ks=K.cuda(), det=det,
                grid=grid, ranges=rng.cuda(), centers=ctr.cuda())


CASES = {
    "cfg0": dict(cfg_id=0),
    "cfg1-8views": dict(cfg_id=1, views=8),
    "cfg2-4views": dict(cfg_id=2, views=4),
    "cfg2-75views": dict(cfg_id=2),
}


@pytest.fixture(scope="module", params=sorted(CASES))
def case(request):
    return request.param, _workload(**CASES[request.param])


def test_wrapper_projection_chain_bit_exact_integers(ref, W, case):
    name, d = case
    import r2s_workloads as wl

    covars, max_s = W.parameter_transform_fwd(d["quats"], d["scales"], wl.SCALE_MIN, wl.SCALE_MAX)
    r_cov, r_max = ref.C.parameter_transform_fwd(d["quats"], d["scales"], wl.SCALE_MIN, wl.SCALE_MAX)
    assert torch.equal(covars, r_cov), f"{name}: covars differ ({rel_l2(covars, r_cov):.3e})"
    assert torch.equal(max_s, r_max)
    det = d["det"]
    m2, c2, radii = W.world_to_image_projection_fwd(d["means"], covars, d["viewmats"], d["Ks"], det,
                                                    det, wl.EPS2D, wl.RADIUS_CLIP)
    rm2, rc2, rradii = ref.C.world_to_image_projection_fwd(d["means"], r_cov, d["viewmats"], d["Ks"],
                                                           det, det, wl.EPS2D, wl.RADIUS_CLIP)
    assert torch.equal(m2, rm2), f"{name}: means2d differ"
    assert rel_l2(c2, rc2) < 1e-6
    assert torch.equal(radii, rradii), f"{name}: {(radii != rradii).sum().item()} radii differ"
    conics, mus = W.conics_mu_fwd(c2, wl.EPS2D)
    rconics, rmus = ref.C.conics_mu_fwd(rc2, wl.EPS2D)
    assert rel_l2(conics, rconics) < REL_L2_F32 and rel_l2(mus, rmus) < REL_L2_F32
    ntx = nty = (det + wl.IMG_TILE - 1) // wl.IMG_TILE
    C = d["viewmats"].shape[0]
    tpg, ids, fids = W.isect_tiles(m2, radii, wl.IMG_TILE, ntx, nty)
    rtpg, rids, rfids = ref.C.isect_tiles(rm2, rradii, wl.IMG_TILE, ntx, nty)
    assert torch.equal(tpg, rtpg)
    assert torch.equal(ids, rids), f"{name}: sorted keys differ"
    assert torch.equal(fids, rfids), f"{name}: sorted flatten ids differ"
    offs = W.isect_offset_encode(ids, C, ntx, nty)
    roffs = ref.C.isect_offset_encode(rids, C, ntx, nty)
    assert torch.equal(offs, roffs)
    # non-rect radii layout [C, N]
    sq = radii.amax(-1).contiguous()
    tpg2, ids2, fids2 = W.isect_tiles(m2, sq, wl.IMG_TILE, ntx, nty)
    rtpg2, rids2, rfids2 = ref.C.isect_tiles(rm2, sq, wl.IMG_TILE, ntx, nty)
    assert torch.equal(tpg2, rtpg2) and torch.equal(ids2, rids2) and torch.equal(fids2, rfids2)


def test_wrapper_volume_chain_bit_exact_integers(ref, W, case):
    name, d = case
    import r2s_workloads as wl

    covars, max_s = W.parameter_transform_fwd(d["quats"], d["scales"], wl.SCALE_MIN, wl.SCALE_MAX)
    G = d["grid"]
    m3, c3, r3 = W.world_to_volume_mapping_fwd(d["means"], covars, max_s, d["ranges"], d["centers"],
                                               G, G, G, wl.EPS3D, wl.RADIUS_CLIP)
    rm3, rc3, rr3 = ref.C.world_to_volume_mapping_fwd(d["means"], covars, max_s, d["ranges"],
                                                      d["centers"], G, G, G, wl.EPS3D,
                                                      wl.RADIUS_CLIP)
    assert torch.equal(m3, rm3)
    assert rel_l2(c3, rc3) < 1e-6
    assert torch.equal(r3, rr3), f"{name}: {(r3 != rr3).sum().item()} 3D radii differ"
    nt = (G + wl.VOL_TILE - 1) // wl.VOL_TILE
    tpg, ids, fids = W.isect_tiles_3d(m3, r3, wl.VOL_TILE, nt, nt, nt)
    rtpg, rids, rfids = ref.C.isect_tiles_3d(rm3, rr3, wl.VOL_TILE, nt, nt, nt)
    assert torch.equal(tpg, rtpg)
    assert torch.equal(ids, rids)
    assert torch.equal(fids, rfids)
    offs = W.isect_offset_encode_3d(ids, nt, nt, nt)
    roffs = ref.C.isect_offset_encode_3d(rids, nt, nt, nt)
    assert torch.equal(offs, roffs)
    vol = W.voxelize_to_voxels_fwd(m3, c3, max_s * 0 + 0.5, offs, fids, G, G, G, wl.VOL_TILE)
    rvol = ref.C.voxelize_to_voxels_fwd(rm3, rc3, max_s * 0 + 0.5, roffs, rfids, G, G, G,
                                        wl.VOL_TILE)
    assert rel_l2(vol, rvol) < REL_L2_F32


@pytest.mark.parametrize("mode", ["primitive", "pixel"])
def test_wrapper_raster_and_voxel_backward(ref, W, case, mode):
    name, d = case
    import r2s_workloads as wl

    covars, max_s, opac = ref.prepare(d["quats"], d["scales"], d["opac"], wl.SCALE_MIN, wl.SCALE_MAX)
    det = d["det"]
    p = ref.rasterize_forward(d["means"], covars, opac, d["viewmats"], d["Ks"], det, det,
                              wl.IMG_TILE, wl.EPS2D, wl.RADIUS_CLIP)
    img = W.rasterize_to_pixels_fwd(p["means2d"], p["conics"], p["opacity"], p["mus"],
                                    p["tile_offsets"], p["flatten_ids"], det, det, wl.IMG_TILE)
    assert rel_l2(img, p["output"]) < REL_L2_F32
    g = torch.Generator(device="cuda").manual_seed(5)
    v_img = torch.randn(p["output"].shape, generator=g, device="cuda")
    args = (p["means2d"], p["conics"], p["opacity"], p["mus"], p["tile_offsets"])
    if mode == "primitive":
        mine = W.rasterize_to_pixels_bwd_per_gaussian(*args, p["isect_ids"], p["flatten_ids"], v_img,
                                                      det, det, wl.IMG_TILE, True)
        theirs = ref.C.rasterize_to_pixels_bwd_per_gaussian(*args, p["isect_ids"], p["flatten_ids"],
                                                            v_img, det, det, wl.IMG_TILE, True)
    else:
        mine = W.rasterize_to_pixels_bwd(*args, p["flatten_ids"], v_img, det, det, wl.IMG_TILE, True)
        theirs = ref.C.rasterize_to_pixels_bwd(*args, p["flatten_ids"], v_img, det, det,
                                               wl.IMG_TILE, True)
    for k, (a, b) in enumerate(zip(mine, theirs)):
        assert rel_l2(a, b) < REL_L2_F32, f"{name}/{mode}: raster grad {k} rel-L2 {rel_l2(a, b):.3e}"
    # downstream chain on identical cotangents
    v_cov = W.conics_mu_bwd(p["cov2d"], p["eps2d"], p["conics"], p["mus"], theirs[2], theirs[4])
    r_vcov = ref.C.conics_mu_bwd(p["cov2d"], p["eps2d"], p["conics"], p["mus"], theirs[2], theirs[4])
    assert rel_l2(v_cov, r_vcov) < REL_L2_F32
    vm, vc = W.world_to_image_projection_bwd(d["means"], covars, d["viewmats"], d["Ks"], det, det,
                                             theirs[1], r_vcov)
    rvm, rvc = ref.C.world_to_image_projection_bwd(d["means"], covars, d["viewmats"], d["Ks"], det,
                                                   det, theirs[1], r_vcov)
    assert rel_l2(vm, rvm) < REL_L2_F32 and rel_l2(vc, rvc) < REL_L2_F32
    vq, vs = W.parameter_transform_bwd(d["quats"], d["scales"], wl.SCALE_MIN, wl.SCALE_MAX, rvc)
    rvq, rvs = ref.C.parameter_transform_bwd(d["quats"], d["scales"], wl.SCALE_MIN, wl.SCALE_MAX, rvc)
    assert rel_l2(vq, rvq) < REL_L2_F32 and rel_l2(vs, rvs) < REL_L2_F32

    G = d["grid"]
    v = ref.voxelize_forward(d["means"], covars, max_s, opac, d["ranges"], d["centers"], G, G, G,
                             wl.VOL_TILE, wl.EPS3D, wl.RADIUS_CLIP)
    v_vol = torch.randn(v["output"].shape, generator=g, device="cuda")
    vargs = (v["means3d"], v["conics"], v["opacity"], v["tile_offsets"])
    if mode == "primitive":
        mine = W.voxelize_to_voxels_bwd_per_gaussian(*vargs, v["isect_ids"], v["flatten_ids"], v_vol,
                                                     G, G, G, wl.VOL_TILE)
        theirs = ref.C.voxelize_to_voxels_bwd_per_gaussian(*vargs, v["isect_ids"], v["flatten_ids"],
                                                           v_vol, G, G, G, wl.VOL_TILE)
    else:
        mine = W.voxelize_to_voxels_bwd(*vargs, v["flatten_ids"], v_vol, G, G, G, wl.VOL_TILE)
        theirs = ref.C.voxelize_to_voxels_bwd(*vargs, v["flatten_ids"], v_vol, G, G, G, wl.VOL_TILE)
    for k, (a, b) in enumerate(zip(mine, theirs)):
        assert rel_l2(a, b) < REL_L2_F32, f"{name}/{mode}: voxel grad {k} rel-L2 {rel_l2(a, b):.3e}"
    vm3, vc3 = W.world_to_volume_mapping_bwd(d["means"], covars, d["ranges"], d["centers"], G, G, G,
                                             wl.EPS3D, theirs[0], theirs[1])
    rvm3, rvc3 = ref.C.world_to_volume_mapping_bwd(d["means"], covars, d["ranges"], d["centers"], G,
                                                   G, G, wl.EPS3D, theirs[0], theirs[1])
    assert rel_l2(vm3, rvm3) < REL_L2_F32 and rel_l2(vc3, rvc3) < REL_L2_F32


def test_fused_op_layer_matches_reference_pipeline(ref, case):
    """The r2splat.ops training path (fused float32 kernels) against the
    reference op-layer call sequence on the reference build."""
    name, d = case
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    det, G = d["det"], d["grid"]
    params = {k: d[k].clone().requires_grad_(True) for k in ("means", "quats", "scales", "opac")}
    state = E.prepare_explicit_gaussians(params["quats"], params["scales"], params["opac"],
                                         scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(state, params["means"], d["viewmats"], d["Ks"], img_w=det, img_h=det,
                               tile_size=wl.IMG_TILE, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                               absgrad=True)
    vres = E.explicit_voxelize(state, params["means"], d["ranges"], d["centers"], dim2=G, dim1=G,
                               dim0=G, tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                               radius_clip=wl.RADIUS_CLIP)
    covars, max_s, opac = ref.prepare(d["quats"], d["scales"], d["opac"], wl.SCALE_MIN, wl.SCALE_MAX)
    assert torch.equal(state.covars, covars)
    # torch.nn.functional.softplus in float, bit for bit (r2s_precise.cu)
    assert torch.equal(state.opacities, opac)
    p = ref.rasterize_forward(d["means"], covars, opac, d["viewmats"], d["Ks"], det, det,
                              wl.IMG_TILE, wl.EPS2D, wl.RADIUS_CLIP)
    v = ref.voxelize_forward(d["means"], covars, max_s, opac, d["ranges"], d["centers"], G, G, G,
                             wl.VOL_TILE, wl.EPS3D, wl.RADIUS_CLIP)
    pb = state.projection.buffers
    vb = state.voxel.buffers
    assert torch.equal(res.radii, p["radii"])
    assert torch.equal(res.means2d.detach(), p["means2d"])
    assert torch.equal(pb.tile_offsets, p["tile_offsets"])
    assert torch.equal(pb.flatten_ids, p["flatten_ids"])
    assert torch.equal(vres.radii, v["radii"])
    assert torch.equal(vb.tile_offsets, v["tile_offsets"])
    assert torch.equal(vb.flatten_ids, v["flatten_ids"])
    assert rel_l2(res.image, p["output"]) < REL_L2_F32
    assert rel_l2(vres.volume, v["output"]) < REL_L2_F32

    g = torch.Generator(device="cuda").manual_seed(7)
    v_img = torch.randn(res.image.shape, generator=g, device="cuda")
    v_vol = torch.randn(vres.volume.shape, generator=g, device="cuda")
    (res.image * v_img).sum().backward()
    (vres.volume * v_vol).sum().backward()
    E.explicit_backward(state, params["means"], params["quats"], params["scales"], params["opac"])
    theirs = ref.explicit_backward(p, v_img, v, v_vol, d["means"], d["quats"], d["scales"], d["opac"],
                                   covars, opac, wl.SCALE_MIN, wl.SCALE_MAX, absgrad=True)
    # every case at the plain bar: the raster backward decides the pixels at
    # the cut-off exactly like the reference (ref_keep2d) and the voxel
    # statistics are float64 sums
    for key, pk in (("means", "means"), ("quats", "quats"), ("scales", "scales"),
                    ("opac", "opacities")):
        e = rel_l2(params[key].grad, theirs[pk])
        assert e < REL_L2_F32, f"{name}: grad {key} rel-L2 {e:.3e}"
    assert rel_l2(res.means2d.grad, theirs["means2d"]) < REL_L2_F32
    assert rel_l2(res.means2d.absgrad, theirs["means2d_abs"]) < REL_L2_F32


def _float64_gradients(ref, d, p, v_img, v, v_vol, covars):
    """Parameter gradients evaluated in float64 by the reference's own double
    kernels from the float32 forward values and the float32 binning (the
    primitive backward of RasterizeToPixelsBwd.cu / VoxelizeToVoxelsBwd.cu and
    the reference VJP chain of r2splat/ops/explicit.py:233-385)."""
    import r2s_workloads as wl

    C = ref.C
    f8 = torch.float64
    det = d["det"]
    G = d["grid"]
    means, cov = d["means"].to(f8), covars.to(f8)
    if p is None:  # volume gradient only
        v_means = torch.zeros_like(means)
        v_cov = torch.zeros_like(cov)
        v_opac = torch.zeros(means.shape[0], dtype=f8, device=means.device)
    else:
        v_abs, v_m2, v_con, v_op, v_mu = C.rasterize_to_pixels_bwd_per_gaussian(
            p["means2d"].to(f8), p["conics"].to(f8), p["opacity"].to(f8), p["mus"].to(f8),
            p["tile_offsets"], p["isect_ids"], p["flatten_ids"], v_img.to(f8), det, det,
            wl.IMG_TILE, False)
        v_c2 = C.conics_mu_bwd(p["cov2d"].to(f8), wl.EPS2D, p["conics"].to(f8), p["mus"].to(f8),
                               v_con.contiguous(), v_mu.contiguous())
        v_means, v_cov = C.world_to_image_projection_bwd(means, cov, d["viewmats"].to(f8),
                                                         d["Ks"].to(f8), det, det,
                                                         v_m2.contiguous(), v_c2.contiguous())
        v_opac = v_op.sum(0)
    v_m3, v_c3, v_o3 = C.voxelize_to_voxels_bwd_per_gaussian(
        v["means3d"].to(f8), v["conics"].to(f8), v["opacity"].to(f8), v["tile_offsets"],
        v["isect_ids"], v["flatten_ids"], v_vol.to(f8), G, G, G, wl.VOL_TILE)
    vm3, vc3 = C.world_to_volume_mapping_bwd(means, cov, v["ranges"].to(f8), v["centers"].to(f8),
                                             G, G, G, wl.EPS3D, v_m3.contiguous(),
                                             v_c3.contiguous())
    v_means = v_means + vm3
    v_cov = v_cov + vc3
    v_opac = v_opac + v_o3
    q8, s8 = d["quats"].to(f8), d["scales"].to(f8)
    v_quats, v_scales = C.parameter_transform_bwd(q8, s8, wl.SCALE_MIN, wl.SCALE_MAX,
                                                  v_cov.contiguous())
    v_raw = v_opac * torch.sigmoid(d["opac"].to(f8))
    return {"means": v_means, "quats": v_quats, "scales": v_scales, "opac": v_raw}


def test_fused_op_layer_accumulates_existing_grads(case):
    name, d = case
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    det = d["det"]
    grads = []
    for accumulate in (False, True):
        params = {k: d[k].clone().requires_grad_(True) for k in ("means", "quats", "scales", "opac")}
        if accumulate:
            for t in params.values():
                t.grad = torch.ones_like(t)
        st = E.prepare_explicit_gaussians(params["quats"], params["scales"], params["opac"],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        r = E.explicit_rasterize(st, params["means"], d["viewmats"], d["Ks"], img_w=det, img_h=det,
                                 tile_size=wl.IMG_TILE, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                                 absgrad=False)
        r.image.square().mean().backward()
        E.explicit_backward(st, params["means"], params["quats"], params["scales"], params["opac"])
        grads.append({k: t.grad.clone() for k, t in params.items()})
    for k in grads[0]:
        torch.testing.assert_close(grads[1][k], grads[0][k] + 1.0, rtol=1e-5, atol=1e-6)


def test_fused_voxel_gradients_alone_match_reference(ref, case):
    """Volume-only upstream gradient: the voxel backward chain is compared on
    its own (the projection's upstream gradient is zero)."""
    name, d = case
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    det, G = d["det"], d["grid"]
    params = {k: d[k].clone().requires_grad_(True) for k in ("means", "quats", "scales", "opac")}
    state = E.prepare_explicit_gaussians(params["quats"], params["scales"], params["opac"],
                                         scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(state, params["means"], d["viewmats"], d["Ks"], img_w=det, img_h=det,
                               tile_size=wl.IMG_TILE, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                               absgrad=False)
    vres = E.explicit_voxelize(state, params["means"], d["ranges"], d["centers"], dim2=G, dim1=G,
                               dim0=G, tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                               radius_clip=wl.RADIUS_CLIP)
    g = torch.Generator(device="cuda").manual_seed(11)
    v_vol = torch.randn(vres.volume.shape, generator=g, device="cuda")
    (res.image * 0).sum().backward()
    (vres.volume * v_vol).sum().backward()
    E.explicit_backward(state, params["means"], params["quats"], params["scales"], params["opac"])
    covars, max_s, opac = ref.prepare(d["quats"], d["scales"], d["opac"], wl.SCALE_MIN, wl.SCALE_MAX)
    v = ref.voxelize_forward(d["means"], covars, max_s, opac, d["ranges"], d["centers"], G, G, G,
                             wl.VOL_TILE, wl.EPS3D, wl.RADIUS_CLIP)
    assert rel_l2(vres.volume, v["output"]) < REL_L2_F32
    theirs = ref.explicit_backward(None, None, v, v_vol, d["means"], d["quats"], d["scales"],
                                   d["opac"], covars, opac, wl.SCALE_MIN, wl.SCALE_MAX)
    for key, pk in (("means", "means"), ("quats", "quats"), ("scales", "scales"),
                    ("opac", "opacities")):
        e = rel_l2(params[key].grad, theirs[pk])
        assert e < REL_L2_F32, f"{name}: voxel-only grad {key} rel-L2 {e:.3e}"


def test_explicit_voxelize_z_slab_matches_full_grid_and_reference(ref, case):
    """explicit_voxelize(..., z_layers=(l0, l1)) -- this build's extension for
    a rank's z-slab -- voxelizes the rows of those brick layers of the full
    grid (same records in the same order per brick: bit-identical when both
    launches use the same number of record groups per brick, else equal to
    float rounding, 1e-6, as launches of few records per SM split each
    brick's records over four groups), and its
    backward of a slab gradient equals the backward of the full grid with
    that gradient placed in a zero volume (the same per-brick moments added
    into float64 per-Gaussian sums, so the order of the additions does not
    show: 1e-6), and the reference's at the plain bar (the voxel backward
    decides the cut-off exactly like the reference)."""
    name, d = case
    import r2s_shard as shard
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    G = d["grid"]
    nt = G // wl.VOL_TILE
    l0, l1 = nt // 4, nt // 4 + max(1, nt // 3)
    z0, z1 = shard.slab_rows(l0, l1, wl.VOL_TILE, G)
    g = torch.Generator(device="cuda").manual_seed(13)
    v_slab = torch.randn((z1 - z0, G, G), generator=g, device="cuda")
    v_full = torch.zeros((G, G, G), device="cuda")
    v_full[z0:z1] = v_slab
    vols, grads = [], []
    for layers, v_vol in ((None, v_full), ((l0, l1), v_slab)):
        params = {k: d[k].clone().requires_grad_(True) for k in ("means", "quats", "scales", "opac")}
        st = E.prepare_explicit_gaussians(params["quats"], params["scales"], params["opac"],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        E.explicit_rasterize(st, params["means"], d["viewmats"][:0], d["Ks"][:0], img_w=16,
                             img_h=16, tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                             radius_clip=wl.RADIUS_CLIP, absgrad=False)
        vr = E.explicit_voxelize(st, params["means"], d["ranges"], d["centers"], dim2=G, dim1=G,
                                 dim0=G, tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                                 radius_clip=wl.RADIUS_CLIP, z_layers=layers)
        vols.append(vr.volume.detach())
        vr.volume.grad = v_vol
        E.explicit_backward(st, params["means"], params["quats"], params["scales"], params["opac"])
        grads.append({k: params[k].grad for k in params})
    assert vols[1].shape == (z1 - z0, G, G)
    e = rel_l2(vols[1], vols[0][z0:z1])
    assert e < 1e-6, f"{name}: slab rows vs the full grid rel-L2 {e:.3e}"
    for key in grads[0]:
        e = rel_l2(grads[1][key], grads[0][key])
        assert e < 1e-6, f"{name}: slab grad {key} vs full-grid grad rel-L2 {e:.3e}"
    covars, max_s, opac = ref.prepare(d["quats"], d["scales"], d["opac"], wl.SCALE_MIN,
                                      wl.SCALE_MAX)
    v = ref.voxelize_forward(d["means"], covars, max_s, opac, d["ranges"], d["centers"], G, G,
                             G, wl.VOL_TILE, wl.EPS3D, wl.RADIUS_CLIP)
    theirs = ref.explicit_backward(None, None, v, v_full, d["means"], d["quats"], d["scales"],
                                   d["opac"], covars, opac, wl.SCALE_MIN, wl.SCALE_MAX)
    for key, pk in (("means", "means"), ("quats", "quats"), ("scales", "scales"),
                    ("opac", "opacities")):
        e = rel_l2(grads[1][key], theirs[pk])
        assert e < REL_L2_F32, f"{name}: slab grad {key} rel-L2 {e:.3e}"
    with pytest.raises(ValueError):
        st = E.prepare_explicit_gaussians(d["quats"], d["scales"], d["opac"],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        E.explicit_voxelize(st, d["means"], d["ranges"], d["centers"], dim2=G, dim1=G, dim0=G,
                            tile_size=wl.VOL_TILE, eps3d=wl.EPS3D, radius_clip=wl.RADIUS_CLIP,
                            z_layers=(0, nt + 1))
