"""Training-step rows after the rasterizer backward: the fused Adam step
against torch.optim.Adam (the optimizer the reference builds,
src/models/gaussian_model.py:514-530) and the fused densification
statistics against the reference strategy's _update_state restated in the
oracle (src/strategies/binary_tree.py:305-347)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = {"means": (5000, 3), "quats": (5000, 4), "scales": (5000, 3), "opacities": (5000,)}
LRS = {"means": 1.6e-4, "quats": 1e-3, "scales": 5e-3, "opacities": 5e-2}


def _params(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return {k: torch.randn(s, generator=g, device="cuda") for k, s in SHAPES.items()}


def test_adam_step_matches_torch_adam():
    from r2splat.ops.training import adam_step

    base = _params(0)
    mine = {k: torch.nn.Parameter(v.clone()) for k, v in base.items()}
    ref = {k: torch.nn.Parameter(v.clone()) for k, v in base.items()}
    opt_mine = {k: torch.optim.Adam([{"params": p, "name": k}], lr=LRS[k], eps=1e-15)
                for k, p in mine.items()}
    opt_ref = {k: torch.optim.Adam([{"params": p, "name": k}], lr=LRS[k], eps=1e-15)
               for k, p in ref.items()}
    g = torch.Generator(device="cuda").manual_seed(1)
    for step in range(1, 4):
        for k in SHAPES:
            grad = torch.randn(SHAPES[k], generator=g, device="cuda") * (10.0 ** -step)
            mine[k].grad = grad.clone()
            ref[k].grad = grad.clone()
        adam_step(opt_mine)
        for o in opt_ref.values():
            o.step()
        for k in SHAPES:
            sm, sr = opt_mine[k].state[mine[k]], opt_ref[k].state[ref[k]]
            assert float(sm["step"]) == float(sr["step"]) == step
            torch.testing.assert_close(sm["exp_avg"], sr["exp_avg"], rtol=1e-6, atol=1e-12)
            torch.testing.assert_close(sm["exp_avg_sq"], sr["exp_avg_sq"], rtol=1e-6, atol=1e-18)
            torch.testing.assert_close(mine[k].detach(), ref[k].detach(), rtol=1e-6, atol=1e-7)
    # the state dicts stay interchangeable
    opt_ref["means"].load_state_dict(opt_mine["means"].state_dict())


def test_adam_step_skips_parameters_without_gradient():
    from r2splat.ops.training import adam_step

    p = torch.nn.Parameter(torch.ones(10, device="cuda"))
    opt = torch.optim.Adam([p], lr=0.1, eps=1e-15)
    adam_step(opt)
    assert len(opt.state) == 0 and torch.equal(p.detach(), torch.ones(10, device="cuda"))


def _info(C, N, seed, zero_frac=0.3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    means2d = torch.zeros(C, N, 2, device="cuda")
    means2d.absgrad = torch.rand(C, N, 2, generator=g, device="cuda") * 1e-3
    means2d.grad = torch.randn(C, N, 2, generator=g, device="cuda") * 1e-3
    radii = torch.randint(1, 40, (C, N), generator=g, device="cuda", dtype=torch.int32)
    radii[torch.rand(C, N, generator=g, device="cuda") < zero_frac] = 0
    return {"means2d": means2d, "radii": radii, "width": 512, "height": 384, "n_cameras": C,
            "gaussian_ids": None}


@pytest.mark.parametrize("absgrad", [True, False])
def test_densify_stats_match_strategy_update(absgrad):
    from oracle import r2s_oracle as O
    from r2splat.ops.training import update_densify_state

    C, N = 4, 3000
    mine, ref = {"grad2d": None, "count": None}, {"grad2d": None, "count": None}
    for seed in (3, 4):  # two steps: accumulation
        info = _info(C, N, seed)
        update_densify_state(mine, info, absgrad=absgrad)
        grads = info["means2d"].absgrad if absgrad else info["means2d"].grad
        O.densify_state_update(ref, grads, info["radii"], info["width"], info["height"], C)
    torch.testing.assert_close(mine["grad2d"], ref["grad2d"], rtol=1e-5, atol=1e-9)
    assert torch.equal(mine["count"], ref["count"])


def test_densify_radius_statistic():
    from oracle import r2s_oracle as O
    from r2splat.ops.training import update_densify_state

    # one view: no duplicate ids, the reference's assignment is exact
    info = _info(1, 2000, 5)
    mine, ref = {"grad2d": None, "count": None}, {"grad2d": None, "count": None}
    update_densify_state(mine, info, track_radii=True)
    O.densify_state_update(ref, info["means2d"].absgrad, info["radii"], 512, 384, 1,
                           track_radii=True)
    assert torch.equal(mine["radii"], ref["radii"])
    # several views: the maximum over the views
    info = _info(5, 2000, 6)
    st = {"grad2d": None, "count": None}
    update_densify_state(st, info, track_radii=True)
    want = (info["radii"].float() / 512.0).amax(0)
    assert torch.equal(st["radii"], want)


def _images(C, H, Wd, seed, smooth):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if smooth:  # projection-like: smooth, positive, with structure
        yy = torch.linspace(-1, 1, H, device="cuda")[:, None]
        xx = torch.linspace(-1, 1, Wd, device="cuda")[None, :]
        base = torch.stack([torch.exp(-((xx - 0.2 * c) ** 2 + yy ** 2) * (2 + c)) for c in range(C)])
        r = base + 0.05 * torch.rand(C, H, Wd, generator=g, device="cuda")
        t = base * 0.9 + 0.05 * torch.rand(C, H, Wd, generator=g, device="cuda")
    else:
        r = torch.rand(C, H, Wd, generator=g, device="cuda")
        t = torch.rand(C, H, Wd, generator=g, device="cuda")
    m = (torch.rand(C, H, Wd, generator=g, device="cuda") < 0.3).float()
    return r[..., None], t[..., None], m[..., None]


@pytest.mark.parametrize("smooth", [False, True])
def test_fused_losses_match_reference_loss_computer(smooth):
    from _helpers import rel_l2
    from oracle import r2s_oracle as O
    from r2splat.ops.training import FusedBinaryTreeLossComputer

    C, H, Wd = 3, 70, 45  # tiles with ragged edges
    r, t, m = _images(C, H, Wd, 8, smooth)
    te = t * 1.1
    g = torch.Generator(device="cuda").manual_seed(9)
    vol = torch.rand(1, 12, 10, 9, generator=g, device="cuda")
    w = dict(w_l1=0.8, w_ssim=0.2, w_tv=0.05, w_edge=0.3)
    r_mine = r.clone().requires_grad_(True)
    v_mine = vol.clone().requires_grad_(True)
    mine = FusedBinaryTreeLossComputer(**w)(r_mine, t, m, v_mine, edge_targets=te)
    mine["total"].backward()
    r_ref = r.clone().requires_grad_(True)
    v_ref = vol.clone().requires_grad_(True)
    # the reference formulas in float32 without TF32 convolutions (cuDNN's
    # default TF32 path alone moves the SSIM gradient by ~1e-4)
    tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ref = O.binary_tree_losses(r_ref, t, m, v_ref, edge_targets=te, **w)
        ref["total"].backward()
    finally:
        torch.backends.cudnn.allow_tf32 = tf32
    for k in ("proj_l1", "proj_ssim", "vol_tv", "edge", "total"):
        a, b = float(mine[k].detach()), float(ref[k].detach())
        assert abs(a - b) <= 1e-5 * max(1e-3, abs(b)), k
    assert rel_l2(r_mine.grad, r_ref.grad) < 1e-5, rel_l2(r_mine.grad, r_ref.grad)
    assert rel_l2(v_mine.grad, v_ref.grad) < 1e-6


def test_projection_losses_at_config_scale_against_float64():
    """Full-size detector batch: values and gradient against the reference
    formulas evaluated in float64."""
    from _helpers import rel_l2
    from oracle import r2s_oracle as O
    from r2splat.ops.training import projection_losses

    r, t, m = _images(4, 512, 512, 10, True)
    x = r.clone().requires_grad_(True)
    l1, ssim, edge = projection_losses(x, t, m)
    (0.8 * l1 + 0.2 * (1 - ssim) + 0.3 * edge).backward()
    x64 = r.double().clone().requires_grad_(True)
    t64, m64 = t.double(), m.double()
    ref = (0.8 * torch.abs(x64 - t64).mean()
           + 0.2 * (1 - O.ssim2d(x64.permute(0, 3, 1, 2), t64.permute(0, 3, 1, 2)))
           + 0.3 * (m64 * torch.abs(x64 - t64)).mean())
    ref.backward()
    total = float((0.8 * l1 + 0.2 * (1 - ssim) + 0.3 * edge).detach())
    assert abs(total - float(ref.detach())) < 1e-5 * float(ref.detach())
    assert rel_l2(x.grad, x64.grad) < 1e-5


def test_fused_plain_loss_computer_matches_reference():
    from _helpers import rel_l2
    from oracle import r2s_oracle as O
    from r2splat.ops.training import FusedLossComputer

    r, t, _ = _images(2, 40, 52, 12, True)
    vol = torch.rand(10, 11, 12, device="cuda")
    w = dict(w_l1=0.7, w_ssim=0.3, w_tv=0.1)
    x1, v1 = r.clone().requires_grad_(True), vol.clone().requires_grad_(True)
    FusedLossComputer(**w)(x1, t, v1)["total"].backward()
    x2, v2 = r.clone().requires_grad_(True), vol.clone().requires_grad_(True)
    tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        O.plain_losses(x2, t, v2, **w)["total"].backward()
    finally:
        torch.backends.cudnn.allow_tf32 = tf32
    assert rel_l2(x1.grad, x2.grad) < 1e-5 and rel_l2(v1.grad, v2.grad) < 1e-6


def test_training_step_gradients_match_reference():
    """One training step at config-1 scale: projection of 4 views, a 32^3 TV
    sub-volume, the BinaryTreeLossComputer terms, the explicit backward; ours
    through r2splat.ops, the reference through its kernels and its PyTorch
    loss (TF32 off).  Loss values and parameter gradients must agree."""
    import r2s_workloads as wl
    from _helpers import rel_l2
    from oracle import r2s_oracle as O
    from oracle.ref_harness import ReferencePipeline
    from r2splat.ops import explicit as E
    from r2splat.ops.training import FusedBinaryTreeLossComputer

    cfg = wl.CONFIGS[1]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg))
    vm, K = wl.make_cameras(4, cfg.detector, total=cfg.n_views)
    vm, K = vm.cuda(), K.cuda()
    det, G = cfg.detector, 32
    rng = torch.full((3,), 0.25, device="cuda")
    ctr = torch.tensor([0.05, -0.1, 0.12], device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(21)
    targets = torch.rand(4, det, det, 1, generator=gen, device="cuda") * 0.1
    edge = (torch.rand(4, det, det, 1, generator=gen, device="cuda") < 0.2).float()
    weights = dict(w_l1=0.8, w_ssim=0.2, w_tv=0.05, w_edge=0.1)

    params = {k: t.clone().requires_grad_(True) for k, t in zip(("m", "q", "s", "o"), (m, q, s, o))}
    st = E.prepare_explicit_gaussians(params["q"], params["s"], params["o"],
                                      scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(st, params["m"], vm, K, img_w=det, img_h=det, tile_size=16,
                               eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP, absgrad=True)
    vox = E.explicit_voxelize(st, params["m"], rng, ctr, dim2=G, dim1=G, dim0=G, tile_size=8,
                              eps3d=wl.EPS3D, radius_clip=wl.RADIUS_CLIP)
    mine = FusedBinaryTreeLossComputer(**weights)(res.image[..., None], targets, edge, vox.volume)
    mine["total"].backward()
    E.explicit_backward(st, params["m"], params["q"], params["s"], params["o"])

    R = ReferencePipeline()
    cov, ms, op = R.prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
    p = R.rasterize_forward(m, cov, op, vm, K, det, det, 16, wl.EPS2D, wl.RADIUS_CLIP)
    v = R.voxelize_forward(m, cov, ms, op, rng, ctr, G, G, G, 8, wl.EPS3D, wl.RADIUS_CLIP)
    image = p["output"].detach().requires_grad_(True)
    volume = v["output"].detach().requires_grad_(True)
    tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ref = O.binary_tree_losses(image[..., None], targets, edge, volume, **weights)
        ref["total"].backward()
    finally:
        torch.backends.cudnn.allow_tf32 = tf32
    g = R.explicit_backward(p, image.grad, v, volume.grad, m, q, s, o, cov, op, wl.SCALE_MIN,
                            wl.SCALE_MAX, absgrad=True)
    for k in ("proj_l1", "proj_ssim", "vol_tv", "edge", "total"):
        a, b = float(mine[k].detach()), float(ref[k].detach())
        assert abs(a - b) <= 1e-5 * max(1e-3, abs(b)), (k, a, b)
    assert rel_l2(res.image.grad, image.grad) < 1e-5
    # parameter gradients: the 1e-5 bar, or within 2e-5 and no less accurate
    # than the reference against a float64 evaluation.  The quaternion
    # gradient of this loss is ill-conditioned: measured, the reference's own
    # float32 result lies 1.9e-5 from the float64 evaluation of the same
    # inputs, this build's as far, and the two 1.0e-5 from each other.
    from _helpers import check_grad_accuracy
    from test_gpu_reference import _float64_gradients

    d = dict(det=det, grid=G, means=m, viewmats=vm, Ks=K, quats=q, scales=s, opac=o)
    truth = _float64_gradients(R, d, p, image.grad, v, volume.grad, cov)
    pairs = (("m", "means"), ("q", "quats"), ("s", "scales"), ("o", "opacities"))
    check_grad_accuracy("training step", {rk: params[k].grad for k, rk in pairs},
                        {rk: g[rk] for _, rk in pairs},
                        {rk: truth[tk] for (_, rk), tk in zip(pairs, ("means", "quats", "scales",
                                                                       "opac"))})


def _render_step(seed, densify=None, with_image_grad=True):
    """One explicit render of a small scene (3 views, 128^2, + a 32^3 volume)
    and its explicit backward; returns the raw parameters and the render."""
    import r2s_workloads as wl
    from r2splat.ops import explicit as E

    cfg = wl.CONFIGS[0]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg, n=3000, seed=seed))
    vm, K = (t.cuda() for t in wl.make_cameras(3, 128))
    params = [t.clone().requires_grad_(True) for t in (m, q, s, o)]
    st = E.prepare_explicit_gaussians(params[1], params[2], params[3], scale_min=wl.SCALE_MIN,
                                      scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(st, params[0], vm, K, img_w=128, img_h=128, tile_size=16,
                               eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP, absgrad=True)
    vox = E.explicit_voxelize(st, params[0], torch.ones(3, device="cuda"),
                              torch.zeros(3, device="cuda"), dim2=32, dim1=32, dim0=32,
                              tile_size=8, eps3d=wl.EPS3D, radius_clip=wl.RADIUS_CLIP)
    g = torch.Generator(device="cuda").manual_seed(seed + 100)
    if with_image_grad:
        (res.image * torch.randn(res.image.shape, generator=g, device="cuda")).sum().backward()
    (vox.volume * torch.randn(vox.volume.shape, generator=g, device="cuda")).sum().backward()
    E.explicit_backward(st, *params, densify=densify)
    return params, res


def _explicit_outputs(st, params, raster_stats, densify_args):
    """One fused explicit backward from fixed raster statistics."""
    from r2splat.cuda import _wrapper as W

    pb = st.projection.buffers
    C, N = pb.means2d.shape[:2]
    v2 = torch.empty((C, N, 2), device="cuda")
    va = torch.empty((C, N, 2), device="cuda")
    outs = [torch.empty(p.shape, device="cuda") for p in params]
    W.fused_explicit_backward(*(p.detach() for p in params), st.scale_min, st.scale_max,
                              pb.viewmats, pb.Ks, pb.img_w, pb.img_h, pb.eps2d, raster_stats,
                              v2 if raster_stats is not None else None,
                              va if raster_stats is not None else None, None, None, 0, 0, 0,
                              0.0, None, False, outs, densify=densify_args)
    return outs, v2, va


@pytest.mark.parametrize("absgrad", [True, False])
@pytest.mark.parametrize("with_image_grad", [True, False])
def test_fused_densify_equals_separate_pass(absgrad, with_image_grad):
    """From the same raster statistics, the fused entry point gives
    bit-identical parameter gradients and densification statistics to the
    plain explicit backward followed by update_densify_state (the raster
    backward itself sums with float atomics, so two renders differ in the
    last bits and the comparison starts after it)."""
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W
    from r2splat.ops import explicit as E
    from r2splat.ops.training import DensifyAccumulator, update_densify_state

    cfg = wl.CONFIGS[0]
    m, q, s_, o = (t.cuda() for t in wl.make_gaussians(cfg, n=3000, seed=21))
    vm, K = (t.cuda() for t in wl.make_cameras(3, 128))
    params = [t.clone().requires_grad_(True) for t in (m, q, s_, o)]
    st = E.prepare_explicit_gaussians(params[1], params[2], params[3], scale_min=wl.SCALE_MIN,
                                      scale_max=wl.SCALE_MAX)
    res = E.explicit_rasterize(st, params[0], vm, K, img_w=128, img_h=128, tile_size=16,
                               eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP, absgrad=True)
    pb = st.projection.buffers
    C, N = pb.means2d.shape[:2]
    stats = None
    if with_image_grad:
        g = torch.Generator(device="cuda").manual_seed(5)
        v_img = torch.randn(res.image.shape, generator=g, device="cuda")
        stats = W.fused_raster_bwd(pb.splats, pb.tile_offsets, pb.flatten_ids, v_img, C, N,
                                   128, 128, 16, pb.tile_offsets.size(2), pb.tile_offsets.size(1),
                                   True)
    sep, fused = {"grad2d": None, "count": None}, {"grad2d": None, "count": None}
    for _ in range(2):  # two steps: accumulation
        outs_a, v2, va = _explicit_outputs(st, params, stats, None)
        means2d = torch.zeros(C, N, 2, device="cuda")
        means2d.grad = v2 if stats is not None else torch.zeros_like(v2)
        means2d.absgrad = va if stats is not None else torch.zeros_like(va)
        info = {"means2d": means2d, "radii": res.radii.amax(-1), "width": 128, "height": 128,
                "n_cameras": C}
        update_densify_state(sep, info, absgrad=absgrad, track_radii=True)
        acc = DensifyAccumulator(fused, absgrad=absgrad, track_radii=True)
        outs_b, _, _ = _explicit_outputs(st, params, stats,
                                         acc.launch_args(res.radii.contiguous(), 128, 128))
        for a, b in zip(outs_a, outs_b):
            assert torch.equal(a, b)
    for key in ("grad2d", "count", "radii"):
        assert torch.equal(sep[key], fused[key]), key
    assert fused["count"].max() > 0
    if with_image_grad:
        assert fused["grad2d"].max() > 0
    else:
        assert fused["grad2d"].max() == 0


def test_explicit_backward_densify_keyword():
    """explicit_backward(densify=...) on two renders of the same scene: the
    statistics agree with the separate pass to float rounding, the counts
    exactly."""
    from r2splat.ops.training import DensifyAccumulator, update_densify_state

    sep, fused = {"grad2d": None, "count": None}, {"grad2d": None, "count": None}
    p_sep, r_sep = _render_step(21)
    update_densify_state(sep, {"means2d": r_sep.means2d, "radii": r_sep.radii.amax(-1),
                               "width": 128, "height": 128, "n_cameras": 3}, absgrad=True)
    p_fus, r_fus = _render_step(21, DensifyAccumulator(fused, absgrad=True))
    for a, b in zip(p_sep, p_fus):
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-4, atol=1e-5)
    assert torch.equal(sep["count"], fused["count"])
    torch.testing.assert_close(sep["grad2d"], fused["grad2d"], rtol=1e-4, atol=1e-6)


def test_fused_densify_without_screen_gradients():
    from r2splat.ops.training import DensifyAccumulator

    a, b = {"grad2d": None, "count": None}, {"grad2d": None, "count": None}
    _, ra = _render_step(23, DensifyAccumulator(a))
    _, rb = _render_step(23, DensifyAccumulator(b, store_screen_grads=False))
    assert rb.means2d.grad is None and getattr(rb.means2d, "absgrad", None) is None
    assert ra.means2d.absgrad is not None
    assert torch.equal(a["count"], b["count"])
    torch.testing.assert_close(a["grad2d"], b["grad2d"], rtol=1e-4, atol=1e-6)


def test_fused_densify_argument_errors():
    from r2splat.ops.training import DensifyAccumulator

    with pytest.raises(RuntimeError, match="must be contiguous float32"):
        _render_step(24, DensifyAccumulator({"grad2d": torch.zeros(5, device="cuda"),
                                             "count": None}))
