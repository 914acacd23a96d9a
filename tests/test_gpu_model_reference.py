"""Drop-in check under the reference's own model class.

The reference's ``GaussianModel`` (src/models/gaussian_model.py:280-492),
unchanged, is executed twice in one process (oracle/ref_stock.py): once with
its ``r2splat`` imports bound to this repository's package, once bound to the
reference's own op layer (r2splat/ops, unchanged) over the reference's CUDA
build (oracle/_ref).  Both instances get the same raw parameters and drive
``prepare_gaussians`` / ``rasterize`` / ``voxelize`` / ``backward_explicit``
as the trainers do (src/trainers/binary_tree.py:159-194): renders, info,
volumes and the parameters' ``.grad`` are compared.  Integer outputs must be
identical, floating-point ones within rel-L2 1e-5.
"""
import math

import pytest
import torch

from _helpers import REL_L2_F32, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def models():
    from oracle import ref_stock

    assert ref_stock.stock_available(), "baseline/_ref or oracle/_ref missing"
    return {b: ref_stock.load_gaussian_model(b) for b in ("ours", "stock")}


def _workload(cfg_id, views=None, n=None):
    import r2s_workloads as wl

    cfg = wl.CONFIGS[cfg_id]
    views = cfg.n_views if views is None else views
    m, q, s, o = wl.make_gaussians(cfg, n=n)
    # camera-to-world matrices of the orbit (the model inverts them itself)
    c2w = torch.stack([wl.camtoworld(2 * math.pi * k / cfg.n_views)
                       for k in range(views)]).float()
    _, Ks = wl.make_cameras(views, cfg.detector, total=cfg.n_views)
    bbox = torch.tensor([[-0.5, -0.5, -0.5], [0.5, 0.5, 0.5]])
    return dict(params=(m, q, s, o), c2w=c2w.cuda(), Ks=Ks.cuda(), det=cfg.detector,
                grid=cfg.grid, bbox=bbox)


def _build(mod, d, mode):
    import r2s_workloads as wl

    gm = mod.GaussianModel(device="cuda", min_scale=wl.SCALE_MIN, max_scale=wl.SCALE_MAX,
                           scale_eps=1e-5, eps2d=wl.EPS2D, eps3d=wl.EPS3D,
                           img_tile_size=wl.IMG_TILE, vol_tile_size=wl.VOL_TILE,
                           img_radius_clip=wl.RADIUS_CLIP, vol_radius_clip=wl.RADIUS_CLIP,
                           backward_mode=mode)
    m, q, s, o = d["params"]
    gm.means = torch.nn.Parameter(m.cuda().clone())
    gm.quats = torch.nn.Parameter(q.cuda().clone())
    gm.scales = torch.nn.Parameter(s.cuda().clone())
    gm.opacities = torch.nn.Parameter(o.cuda().clone())
    return gm


def _train_step(gm, d, v_r, v_v):
    G = d["grid"]
    state = gm.prepare_gaussians(explicit=True)
    renders, info = gm.rasterize(d["c2w"], d["Ks"], d["det"], d["det"], absgrad=True,
                                 gaussian_state=state)
    vol = gm.voxelize((G, G, G), d["bbox"], gaussian_state=state)
    ((renders * v_r).sum() + (vol * v_v).sum()).backward()
    gm.backward_explicit(state)
    return renders.detach(), info, vol.detach()


CASES = {"cfg0": dict(cfg_id=0), "cfg1-8views": dict(cfg_id=1, views=8)}


@pytest.mark.parametrize("mode", ["primitive", "pixel"])
@pytest.mark.parametrize("case", sorted(CASES))
def test_reference_model_class_training_step(models, case, mode):
    d = _workload(**CASES[case])
    ours = _build(models["ours"], d, mode)
    theirs = _build(models["stock"], d, mode)
    C, det, G = d["c2w"].shape[0], d["det"], d["grid"]
    g = torch.Generator(device="cuda").manual_seed(21)
    v_r = torch.randn((C, det, det, 1), generator=g, device="cuda")
    v_v = torch.randn((G, G, G, 1), generator=g, device="cuda")
    r_o, info_o, vol_o = _train_step(ours, d, v_r, v_v)
    r_t, info_t, vol_t = _train_step(theirs, d, v_r, v_v)
    assert r_o.shape == r_t.shape == (C, det, det, 1)
    assert vol_o.shape == vol_t.shape == (G, G, G, 1)
    assert rel_l2(r_o, r_t) < REL_L2_F32, f"{case}: renders rel-L2 {rel_l2(r_o, r_t):.3e}"
    assert rel_l2(vol_o, vol_t) < REL_L2_F32, f"{case}: volume rel-L2 {rel_l2(vol_o, vol_t):.3e}"
    assert torch.equal(info_o["radii"], info_t["radii"])
    assert torch.equal(info_o["means2d"].detach(), info_t["means2d"].detach())
    assert torch.equal(info_o["gaussian_ids"], info_t["gaussian_ids"])
    for k in ("width", "height", "n_cameras"):
        assert info_o[k] == info_t[k]
    e = rel_l2(info_o["means2d"].grad, info_t["means2d"].grad)
    assert e < REL_L2_F32, f"{case}/{mode}: means2d.grad rel-L2 {e:.3e}"
    e = rel_l2(info_o["means2d"].absgrad, info_t["means2d"].absgrad)
    assert e < REL_L2_F32, f"{case}/{mode}: means2d.absgrad rel-L2 {e:.3e}"
    for name in ("means", "quats", "scales", "opacities"):
        a, b = getattr(ours, name).grad, getattr(theirs, name).grad
        e = rel_l2(a, b)
        assert e < REL_L2_F32, f"{case}/{mode}: {name}.grad rel-L2 {e:.3e}"


def test_reference_model_class_inference_and_options(models):
    d = _workload(cfg_id=1, views=4)
    ours = _build(models["ours"], d, "primitive")
    theirs = _build(models["stock"], d, "primitive")
    G = d["grid"]
    with torch.no_grad():
        outs = []
        for gm in (ours, theirs):
            st = gm.prepare_gaussians()
            r, info = gm.rasterize(d["c2w"], d["Ks"], d["det"], d["det"], gaussian_state=st)
            v = gm.voxelize((G, G, G), d["bbox"], gaussian_state=st)
            # a state is built per call when none is given
            r2, _ = gm.rasterize(d["c2w"], d["Ks"], d["det"], d["det"])
            outs.append((r, info, v, r2, gm.voxelize((G, G, G), None)))
    (r_o, i_o, v_o, r2_o, none_o), (r_t, i_t, v_t, r2_t, none_t) = outs
    assert rel_l2(r_o, r_t) < REL_L2_F32 and rel_l2(v_o, v_t) < REL_L2_F32
    assert torch.equal(r_o, r2_o) and torch.equal(i_o["radii"], i_t["radii"])
    assert none_o is None and none_t is None
    # the model's option errors reach the caller the same way over both backends
    for kwargs, exc in (({"packed": True}, ValueError), ({"sparse_grad": True}, ValueError),
                        ({"rasterize_mode": "antialiased"}, ValueError),
                        ({"camera_model": "ortho"}, ValueError), ({"foo": 1}, TypeError)):
        msgs = []
        for gm in (ours, theirs):
            with pytest.raises(exc) as ei:
                gm.rasterize(d["c2w"], d["Ks"], d["det"], d["det"], **kwargs)
            msgs.append(str(ei.value))
        assert msgs[0] == msgs[1]
    # an explicit state is single-use in both op layers
    for gm in (ours, theirs):
        st = gm.prepare_gaussians(explicit=True)
        gm.rasterize(d["c2w"], d["Ks"], d["det"], d["det"], gaussian_state=st)
        with pytest.raises(RuntimeError):
            gm.rasterize(d["c2w"], d["Ks"], d["det"], d["det"], gaussian_state=st)
