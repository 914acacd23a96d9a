"""Parity at benchmark config 3 (2M Gaussians, 30 % on a thin shell, 768^2
detector, 512^3 grid) against the live reference build (oracle/_ref).

Projection: the first 40 views of the 100-view orbit hold about 4e9
intersection records, past the int32 tile offsets of one binning
(r2splat/cuda/csrc/IsectTiles.cpp:95-114, the reference's own limit).  The
op layer then bins and rasterizes contiguous view batches
(``plan_view_batches``).  The reference is run on the same view ranges, batch
by batch, as its callers must: sorted flatten ids and tile offsets are
compared bit for bit per batch, radii and means2d per view, images within
rel-L2 1e-5, and the parameter gradients summed over the batches.

Voxelization: one z-slab of the 8-slab split of the 512^3 grid (the
multi-GPU sharding) is binned in the global key space and voxelized alone;
its flatten ids and (rebased) tile offsets must equal the reference's for the
same brick layers, its volume the same rows of the reference volume, and
the gradients of an upstream gradient on the slab the reference's.
"""
import pytest
import torch

from _helpers import REL_L2_F32, rel_l2

pytestmark = pytest.mark.gpu

VIEWS = 40


@pytest.fixture(scope="module")
def ref():
    from oracle.ref_harness import REF_SO, ReferencePipeline
    import os

    assert os.path.exists(REF_SO), "reference build missing: run python oracle/build_ref.py"
    return ReferencePipeline()


@pytest.fixture(scope="module")
def cfg3():
    import r2s_workloads as wl

    cfg = wl.CONFIGS[3]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg))
    return cfg, dict(means=m, quats=q, scales=s, opac=o)


def test_config3_view_batches_match_reference_batches(ref, cfg3):
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    cfg, d = cfg3
    det = cfg.detector
    vm, K = wl.make_cameras(VIEWS, det, total=cfg.n_views)
    vm, K = vm.cuda(), K.cuda()
    params = {k: d[k].clone().requires_grad_(True) for k in ("means", "quats", "scales", "opac")}
    st = E.prepare_explicit_gaussians(params["quats"], params["scales"], params["opac"],
                                      scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(st, params["means"], vm, K, img_w=det, img_h=det,
                               tile_size=wl.IMG_TILE, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                               absgrad=True)
    pb = st.projection.buffers
    assert pb.view_batches is not None and len(pb.view_batches) >= 2, \
        "config 3 must exceed one int32 binning"
    n_total = sum(ids.numel() for _, _, ids in pb.view_batches)
    assert n_total > 2 ** 31 - 1
    g = torch.Generator(device="cuda").manual_seed(33)
    v_img = torch.randn(res.image.shape, generator=g, device="cuda")
    (res.image * v_img).sum().backward()
    E.explicit_backward(st, params["means"], params["quats"], params["scales"], params["opac"])
    ours = {k: params[k].grad for k in params}

    covars, _, opac = ref.prepare(d["quats"], d["scales"], d["opac"], wl.SCALE_MIN, wl.SCALE_MAX)
    assert torch.equal(st.covars, covars)
    theirs = {k: torch.zeros_like(d[k]) for k in params}
    m2_grad = []
    for c0, c1, ids in pb.view_batches:
        p = ref.rasterize_forward(d["means"], covars, opac, vm[c0:c1], K[c0:c1], det, det,
                                  wl.IMG_TILE, wl.EPS2D, wl.RADIUS_CLIP)
        assert torch.equal(ids, p["flatten_ids"]), f"views {c0}:{c1}: flatten ids differ"
        assert torch.equal(pb.tile_offsets[c0:c1], p["tile_offsets"]), \
            f"views {c0}:{c1}: tile offsets differ"
        assert torch.equal(res.radii[c0:c1], p["radii"])
        assert torch.equal(res.means2d[c0:c1].detach(), p["means2d"])
        e = rel_l2(res.image[c0:c1].detach(), p["output"])
        assert e < REL_L2_F32, f"views {c0}:{c1}: image rel-L2 {e:.3e}"
        gb = ref.explicit_backward(p, v_img[c0:c1], None, None, d["means"], d["quats"],
                                   d["scales"], d["opac"], covars, opac, wl.SCALE_MIN,
                                   wl.SCALE_MAX, absgrad=True)
        for k, pk in (("means", "means"), ("quats", "quats"), ("scales", "scales"),
                      ("opac", "opacities")):
            theirs[k] += gb[pk]
        m2_grad.append((c0, c1, gb["means2d"], gb["means2d_abs"]))
        del p, gb
        torch.cuda.empty_cache()
    for c0, c1, gm2, gabs in m2_grad:
        assert rel_l2(res.means2d.grad[c0:c1], gm2) < REL_L2_F32
        assert rel_l2(res.means2d.absgrad[c0:c1], gabs) < REL_L2_F32
    for k in ours:  # the plain bar (exact cut-off decisions in the raster backward)
        e = rel_l2(ours[k], theirs[k])
        assert e < REL_L2_F32, f"cfg3-40views: grad {k} rel-L2 {e:.3e}"


def test_config3_z_slab_matches_reference_layers(ref, cfg3):
    import r2s_shard as shard
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W

    cfg, d = cfg3
    G = cfg.grid
    nt = (G + wl.VOL_TILE - 1) // wl.VOL_TILE
    rng, ctr = (t.cuda() for t in wl.unit_cube_box())
    m, q, s, o = (d[k] for k in ("means", "quats", "scales", "opac"))
    # slab 3 of the equal 8-slab split (the shell crosses it)
    l0, l1 = 3 * nt // 8, 4 * nt // 8
    z0, z1 = shard.slab_rows(l0, l1, wl.VOL_TILE, G)
    N = m.size(0)
    with torch.no_grad():
        cov, ms, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
        m3, c3, r3, vs, rects, _ = W.fused_map(m, cov, op, rng, ctr, G, G, G, wl.VOL_TILE, nt,
                                               nt, nt, wl.EPS3D, wl.RADIUS_CLIP)
        offs, fids, _ = W.fused_bin(rects, l1 - l0, N, nt * nt, nt, 1, segment_base=l0)
        rows = W.fused_voxel_rows(vs, offs, fids, N, G, G, G, wl.VOL_TILE, nt, nt, nt, l0, l1)
        vol = W.fused_voxel_fwd(vs, offs, fids, N, G, G, G, wl.VOL_TILE, nt, nt, nt, l0, l1,
                                rows=rows)
    covars, max_s, opac = ref.prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
    v = ref.voxelize_forward(m, covars, max_s, opac, rng, ctr, G, G, G, wl.VOL_TILE, wl.EPS3D,
                             wl.RADIUS_CLIP)
    assert torch.equal(r3, v["radii"]) and torch.equal(m3, v["means3d"])
    roffs = v["tile_offsets"]
    start = int(roffs[l0].flatten()[0])
    end = int(roffs[l1].flatten()[0]) if l1 < nt else v["flatten_ids"].numel()
    assert torch.equal(fids, v["flatten_ids"][start:end]), "slab flatten ids differ"
    assert torch.equal(offs.view(l1 - l0, nt, nt), roffs[l0:l1] - start), "slab offsets differ"
    e = rel_l2(vol, v["output"][z0:z1])
    assert e < REL_L2_F32, f"slab volume rel-L2 {e:.3e}"

    g = torch.Generator(device="cuda").manual_seed(34)
    v_slab = torch.randn(vol.shape, generator=g, device="cuda")
    v_full = torch.zeros_like(v["output"])
    v_full[z0:z1] = v_slab
    with torch.no_grad():
        stats = W.fused_voxel_bwd(vs, offs, fids, v_slab, N, G, G, G, wl.VOL_TILE, nt, nt, nt,
                                  l0, l1, rows=rows)
        outs = [torch.empty_like(t) for t in (m, q, s, o)]
        W.fused_explicit_backward(m, q, s, o, wl.SCALE_MIN, wl.SCALE_MAX, None, None, 0, 0,
                                  wl.EPS2D, None, None, None, rng, ctr, G, G, G, wl.EPS3D, stats,
                                  False, outs)
    theirs = ref.explicit_backward(None, None, v, v_full, m, q, s, o, covars, opac, wl.SCALE_MIN,
                                   wl.SCALE_MAX)
    for got, key in zip(outs, ("means", "quats", "scales", "opacities")):
        e = rel_l2(got, theirs[key])
        assert e < REL_L2_F32, f"slab grad {key} rel-L2 {e:.3e}"
