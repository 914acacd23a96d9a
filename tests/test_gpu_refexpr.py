"""Which restatement of the reference's cut-off expression rounds exactly
like the reference's compiled kernels (bt-3dgs_b200/csrc/r2s_refexpr.cuh).

One Gaussian per image, radii covering the whole image, so the reference's
forward (csrc/RasterizeToPixelsFwd.cu:159-179) evaluates every pixel and its
image holds exactly alpha where it keeps the pair and 0 where it drops it.
The probe (tests/refexpr_probe.cu, built here with the library's nvcc
flags) evaluates each variant on the same pixels; the backward's decision
(csrc/RasterizeToPixelsBwd.cu:423-430) is read from v_mus of a one-hot
upstream gradient at each image's pixel nearest the cut-off.  The test
reports every variant's mismatch counts and requires one that matches both
exactly.
"""
import ctypes
import os
import subprocess

import pytest
import torch

from _helpers import REL_L2_F32, ROOT, rel_l2

pytestmark = pytest.mark.gpu

VARIANTS = {0: "source expression", 1: "fma(0.5, fma(a dx, dx, c dy dy), b dx dy)",
            2: "fma(b dx, dy, 0.5 fma(a dx, dx, c dy dy))",
            3: "fma(0.5, fma(c dy, dy, a dx dx), b dx dy)",
            4: "fma(b dx, dy, 0.5 fma(c dy, dy, a dx dx))", 5: "unfused"}


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("probe") / "refexpr_probe.so")
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "r2s_build", os.path.join(ROOT, "bt-3dgs_b200", "build.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    cmd = [b._nvcc(), *b.NVCC_FLAGS, "-shared", "-o", out,
           os.path.join(ROOT, "tests", "refexpr_probe.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    lib = ctypes.CDLL(out)
    lib.probe_alpha2d.restype = ctypes.c_int
    return lib


def _inputs(C, W, seed=0):
    g = torch.Generator().manual_seed(seed)
    m = torch.rand(C, 2, generator=g) * W
    # covariances from random scales (0.3 .. 12 px) and rotations, conic = inverse
    s = torch.exp(torch.empty(C, 2).uniform_(-1.2, 2.5, generator=g))
    th = torch.rand(C, generator=g) * 6.2831853
    R = torch.stack([torch.stack([th.cos(), -th.sin()], -1), torch.stack([th.sin(), th.cos()], -1)],
                    -2)
    cov = R @ torch.diag_embed(s * s) @ R.transpose(-1, -2)
    inv = torch.linalg.inv(cov.double()).float()
    conics = torch.stack([inv[:, 0, 0], inv[:, 0, 1], inv[:, 1, 1]], -1)
    wmu = torch.exp(torch.empty(C).uniform_(-11.0, 0.0, generator=g))  # 1.7e-5 .. 1
    return m, conics, wmu


def test_reference_cut_off_expression_is_reproduced(probe):
    from oracle.ref_harness import ReferencePipeline

    ref = ReferencePipeline()
    C, W = 4096, 64
    m, conics, wmu = _inputs(C, W)
    dev = "cuda"
    m2 = m.reshape(C, 1, 2).contiguous().to(dev)
    con = conics.reshape(C, 1, 3).contiguous().to(dev)
    op = wmu.reshape(C, 1).contiguous().to(dev)
    mus = torch.ones((C, 1), device=dev)  # opacity * mu = wmu exactly
    radii = torch.full((C, 1, 2), 4 * W, dtype=torch.int32, device=dev)
    nt = W // 16
    _, ids, fids = ref.C.isect_tiles(m2, radii, 16, nt, nt)
    offs = ref.C.isect_offset_encode(ids, C, nt, nt)
    img = ref.C.rasterize_to_pixels_fwd(m2, con, op, mus, offs, fids, W, W, 16)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    report = {}
    outs = {}
    for v in VARIANTS:
        out = torch.empty((C, W, W), device=dev)
        rc = probe.probe_alpha2d(v, ctypes.c_void_p(m2.data_ptr()), ctypes.c_void_p(con.data_ptr()),
                                 ctypes.c_void_p(op.data_ptr()), C, W, W,
                                 ctypes.c_void_p(out.data_ptr()), stream)
        assert rc == 0
        torch.cuda.synchronize()
        outs[v] = out
        report[v] = {"value_mismatch": int((out != img).sum()),
                     "decision_mismatch": int(((out != 0) != (img != 0)).sum())}
    # backward decision at each image's pixel nearest the cut-off (by variant 0's sigma)
    sigma_cut = torch.log(op.reshape(C, 1, 1) * 1e5)
    ys, xs = torch.meshgrid(torch.arange(W, device=dev) + 0.5, torch.arange(W, device=dev) + 0.5,
                            indexing="ij")
    dx = xs[None] - m2[:, 0, 0, None, None]
    dy = ys[None] - m2[:, 0, 1, None, None]
    a, b, c = con[:, 0, 0, None, None], con[:, 0, 1, None, None], con[:, 0, 2, None, None]
    sig = 0.5 * (a * dx * dx + c * dy * dy) + b * dx * dy
    near = (sig - sigma_cut).abs().reshape(C, -1).argmin(1)
    v_img = torch.zeros((C, W * W), device=dev)
    v_img[torch.arange(C, device=dev), near] = 1.0
    v_img = v_img.reshape(C, W, W)
    grads = ref.C.rasterize_to_pixels_bwd_per_gaussian(m2, con, op, mus, offs, ids, fids, v_img,
                                                       W, W, 16, False)
    ref_keep = grads[4].reshape(C) != 0  # v_mus = opacity * vis at the one pixel, 0 if dropped
    for v in VARIANTS:
        ours_keep = outs[v].reshape(C, -1)[torch.arange(C, device=dev), near] != 0
        report[v]["bwd_decision_mismatch"] = int((ours_keep != ref_keep).sum())
    print({VARIANTS[k]: r for k, r in report.items()})
    exact = [v for v, r in report.items() if r["value_mismatch"] == 0
             and r["bwd_decision_mismatch"] == 0]
    assert exact, f"no variant reproduces the reference: {report}"


def test_raster_backward_decides_the_cut_off_like_the_reference():
    """The pixels nearest the cut-off, one per image: this build's raster
    backward (the 16x16 kernel: fast test, cut-off band, re-decision with
    ref_keep2d) keeps exactly the pixels the reference's backward keeps.
    Each Gaussian is replicated over K images, each with a one-hot upstream
    gradient at one of its K pixels nearest the cut-off (by a float64
    sigma); v_mu = opacity * vis at that pixel when it is kept, 0 when it is
    dropped -- a decision per image, read from both builds."""
    from oracle.ref_harness import ReferencePipeline
    from r2splat.cuda import _wrapper as Wr

    ref = ReferencePipeline()
    C0, W, K = 4096, 64, 4
    m, conics, wmu = _inputs(C0, W, seed=1)
    dev = "cuda"
    # mu != 1: the reference's alpha rounds (opacity * mu) * vis
    g = torch.Generator().manual_seed(2)
    mus = torch.empty(C0).uniform_(0.3, 1.0, generator=g)
    op = (wmu / mus).clamp(max=1.0)
    rep = lambda t: t.repeat_interleave(K, 0).contiguous().to(dev)  # noqa: E731
    C = C0 * K
    m2 = rep(m).reshape(C, 1, 2)
    con = rep(conics).reshape(C, 1, 3)
    opac = rep(op).reshape(C, 1)
    mu = rep(mus).reshape(C, 1)
    radii = torch.full((C, 1, 2), 4 * W, dtype=torch.int32, device=dev)
    nt = W // 16
    _, ids, fids = ref.C.isect_tiles(m2, radii, 16, nt, nt)
    offs = ref.C.isect_offset_encode(ids, C, nt, nt)
    # K pixels nearest the cut-off of each Gaussian, by a float64 sigma
    f8 = torch.float64
    ys, xs = torch.meshgrid(torch.arange(W, dtype=f8) + 0.5, torch.arange(W, dtype=f8) + 0.5,
                            indexing="ij")
    dx = xs[None] - m[:, 0, None, None].to(f8)
    dy = ys[None] - m[:, 1, None, None].to(f8)
    a, b, c = (conics[:, k, None, None].to(f8) for k in range(3))
    sig = 0.5 * (a * dx * dx + c * dy * dy) + b * dx * dy
    w8 = (op.to(f8) * mus.to(f8))[:, None, None]
    gap = (sig - torch.log(w8 * 1e5)).abs().reshape(C0, -1)
    near = gap.topk(K, dim=1, largest=False).indices.reshape(C)  # [C0 * K]
    v_img = torch.zeros((C, W * W), device=dev)
    v_img[torch.arange(C, device=dev), near.to(dev)] = 1.0
    v_img = v_img.reshape(C, W, W)
    args = (m2, con, opac, mu, offs, ids, fids, v_img, W, W, 16, False)
    theirs = ref.C.rasterize_to_pixels_bwd_per_gaussian(*args)
    mine = Wr.rasterize_to_pixels_bwd_per_gaussian(*args)
    ref_keep = theirs[4].reshape(C) != 0
    our_keep = mine[4].reshape(C) != 0
    # the reference's pixel backward mode decides alike
    pix = ref.C.rasterize_to_pixels_bwd(m2, con, opac, mu, offs, fids, v_img, W, W, 16, False)
    assert torch.equal(pix[4].reshape(C) != 0, ref_keep)
    kept = int(ref_keep.sum())
    assert 0 < kept < C, kept  # both decisions occur among the tested pixels
    assert torch.equal(our_keep, ref_keep), (
        f"{int((our_keep != ref_keep).sum())} of {C} cut-off decisions differ")
    # the kept values: opacity * vis from each build's own exponential (this
    # build's pre-scaled exp2, the reference's __expf)
    e = rel_l2(mine[4].reshape(C)[ref_keep], theirs[4].reshape(C)[ref_keep])
    assert e < REL_L2_F32, e


VARIANTS3D = {0: "source expression",
              1: "X = fma(c d3, d3, fma(a d1, d1, (b d2) d2)); cross products into 0.5 X",
              2: "X = fma(c d3, d3, fma(b d2, d2, (a d1) d1)); cross products into 0.5 X",
              3: "X as 1; fma(0.5, X, (p d1) d2), then the other cross products",
              4: "X as 2; fma(0.5, X, (p d1) d2), then the other cross products",
              5: "unfused"}


def _inputs3d(ncell, seed=0):
    """One Gaussian per 16^3 cell of a (16 ncell)^3 volume, its support (alpha
    >= 1e-6) inside the cell: means within a voxel of the cell centre, axis
    scales 0.4 .. 1.2 voxels, random rotations, opacities 2e-6 .. 1."""
    g = torch.Generator().manual_seed(seed)
    C = ncell ** 3
    idx = torch.arange(C)
    cells = torch.stack([idx % ncell, (idx // ncell) % ncell, idx // (ncell * ncell)], -1) * 16
    m = cells.float() + 8.0 + (torch.rand(C, 3, generator=g) * 2 - 1)
    s = torch.empty(C, 3).uniform_(0.4, 1.2, generator=g)
    q = torch.randn(C, 4, generator=g)
    q = q / q.norm(dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    R = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                     2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                     2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
                    -1).reshape(C, 3, 3)
    cov = R @ torch.diag_embed(s * s) @ R.transpose(-1, -2)
    P = torch.linalg.inv(cov.double()).float()
    conics = torch.stack([P[:, 0, 0], P[:, 0, 1], P[:, 0, 2], P[:, 1, 1], P[:, 1, 2], P[:, 2, 2]],
                         -1)
    opac = torch.exp(torch.empty(C).uniform_(-13.0, 0.0, generator=g))
    return m, conics, opac, cells.int()


def test_reference_voxel_cut_off_expression_is_reproduced(probe):
    """3D: the reference's voxelizer forward with one Gaussian per 16^3 cell
    (csrc/VoxelizeToVoxelsFwd.cu:195-210) holds each Gaussian's alpha or 0 in
    its cell; each variant is evaluated on the same voxels, and the
    backward's decision (csrc/VoxelizeToVoxelsBwd.cu:395-402) is read from
    v_opacity of a one-hot upstream gradient at each cell's voxel nearest the
    cut-off.  Requires a variant that matches both exactly; the reference's
    pixel backward mode decides like its primitive mode."""
    from oracle.ref_harness import ReferencePipeline

    probe.probe_alpha3d.restype = ctypes.c_int
    ref = ReferencePipeline()
    ncell = 16
    G = 16 * ncell
    m, conics, opac, cells = _inputs3d(ncell)
    C = m.size(0)
    dev = "cuda"
    m3, con, op, cl = (t.contiguous().to(dev) for t in (m, conics, opac, cells))
    radii = torch.full((C, 3), 8, dtype=torch.int32, device=dev)
    nt = G // 8
    _, ids, fids = ref.C.isect_tiles_3d(m3, radii, 8, nt, nt, nt)
    offs = ref.C.isect_offset_encode_3d(ids, nt, nt, nt)
    vol = ref.C.voxelize_to_voxels_fwd(m3, con, op, offs, fids, G, G, G, 8)
    # the reference volume cut into the cells: [C, 16, 16, 16] (z, y, x)
    cz, cy, cx = cl[:, 2].long(), cl[:, 1].long(), cl[:, 0].long()
    r16 = torch.arange(16, device=dev)
    zz = (cz[:, None] + r16)[:, :, None, None]
    yy = (cy[:, None] + r16)[:, None, :, None]
    xx = (cx[:, None] + r16)[:, None, None, :]
    ref_cells = vol[zz, yy, xx].reshape(C, -1)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    report, outs = {}, {}
    for v in VARIANTS3D:
        out = torch.empty((C, 4096), device=dev)
        rc = probe.probe_alpha3d(v, ctypes.c_void_p(m3.data_ptr()), ctypes.c_void_p(con.data_ptr()),
                                 ctypes.c_void_p(op.data_ptr()), ctypes.c_void_p(cl.data_ptr()),
                                 C, ctypes.c_void_p(out.data_ptr()), stream)
        assert rc == 0
        torch.cuda.synchronize()
        outs[v] = out
        report[v] = {"value_mismatch": int((out != ref_cells).sum()),
                     "decision_mismatch": int(((out != 0) != (ref_cells != 0)).sum())}
    assert int((ref_cells != 0).sum()) > 0
    # backward decision at each cell's voxel nearest the cut-off (float64 sigma)
    f8 = torch.float64
    gz, gy, gx = torch.meshgrid(r16.to(f8) + 0.5, r16.to(f8) + 0.5, r16.to(f8) + 0.5,
                                indexing="ij")
    d1 = cx.to(f8)[:, None, None, None] + gx[None] - m3[:, 0, None, None, None].to(f8)
    d2 = cy.to(f8)[:, None, None, None] + gy[None] - m3[:, 1, None, None, None].to(f8)
    d3 = cz.to(f8)[:, None, None, None] + gz[None] - m3[:, 2, None, None, None].to(f8)
    k = [con[:, i, None, None, None].to(f8) for i in range(6)]
    sig = (0.5 * (k[0] * d1 * d1 + k[3] * d2 * d2 + k[5] * d3 * d3) + k[1] * d1 * d2
           + k[2] * d1 * d3 + k[4] * d2 * d3)
    cut = torch.log(op.to(f8) * 1e6)[:, None, None, None]
    near = (sig - cut).abs().reshape(C, -1).argmin(1)  # [C], cell-local z*256 + y*16 + x
    v_vol = torch.zeros((G, G, G), device=dev)
    nz, ny, nx = near // 256, (near // 16) % 16, near % 16
    v_vol[cz + nz, cy + ny, cx + nx] = 1.0
    grads = ref.C.voxelize_to_voxels_bwd_per_gaussian(m3, con, op, offs, ids, fids, v_vol, G, G,
                                                      G, 8)
    ref_keep = grads[2].reshape(C) != 0  # v_opacity = vis at the one voxel, 0 if dropped
    # the reference's pixel backward mode decides alike
    pix = ref.C.voxelize_to_voxels_bwd(m3, con, op, offs, fids, v_vol, G, G, G, 8)
    assert torch.equal(pix[2].reshape(C) != 0, ref_keep)
    for v in VARIANTS3D:
        ours_keep = outs[v][torch.arange(C, device=dev), near] != 0
        report[v]["bwd_decision_mismatch"] = int((ours_keep != ref_keep).sum())
    print({VARIANTS3D[k]: r for k, r in report.items()})
    exact = [v for v, r in report.items() if r["value_mismatch"] == 0
             and r["bwd_decision_mismatch"] == 0]
    assert exact, f"no variant reproduces the reference: {report}"


def test_voxel_backward_decides_the_cut_off_like_the_reference():
    """The op layer's voxel backward (the fused 8x8x8 kernel: fast test,
    cut-off band, re-decision with ref_keep3d) keeps exactly the voxels the
    reference's backward keeps.  One Gaussian per 16^3 cell of a 256^3 grid
    (world means at the cell centres, voxel-space scales 0.4 .. 1.2,
    opacities 2e-6 .. 1, a culling radius that bins the whole support); the
    upstream gradient is one-hot at each cell's voxel nearest the Gaussian's
    cut-off (float64 sigma from the reference's conic).  The gradient of a
    raw opacity is sigmoid(raw) * vis at that voxel when it is kept and 0
    when it is dropped: a decision per Gaussian, read from both builds."""
    import r2s_workloads as wl
    from oracle.ref_harness import ReferencePipeline
    from r2splat.ops import explicit as E

    ref = ReferencePipeline()
    G, ncell, dev = 256, 16, "cuda"
    C = ncell ** 3
    g = torch.Generator().manual_seed(3)
    idx = torch.arange(C)
    cells = torch.stack([idx % ncell, (idx // ncell) % ncell, idx // (ncell * ncell)], -1) * 16
    vox_means = cells.float() + 8.0 + (torch.rand(C, 3, generator=g) * 2 - 1)
    means = ((vox_means - G / 2) / G).to(dev)
    scales = wl.inverse_scale(torch.empty(C, 3).uniform_(0.4, 1.2, generator=g) / G).to(dev)
    quats = torch.randn(C, 4, generator=g).to(dev)
    opac = wl.inverse_softplus(torch.exp(torch.empty(C).uniform_(-13.1, 0.0, generator=g))).to(dev)
    rng, ctr = (t.to(dev) for t in wl.unit_cube_box())
    clip = 8.0
    covars, max_s, op = ref.prepare(quats, scales, opac, wl.SCALE_MIN, wl.SCALE_MAX)
    v = ref.voxelize_forward(means, covars, max_s, op, rng, ctr, G, G, G, wl.VOL_TILE, wl.EPS3D,
                             clip)
    f8 = torch.float64
    m3, k = v["means3d"].to(f8), v["conics"].to(f8)
    cl = cells.to(dev)
    r16 = torch.arange(16, device=dev, dtype=f8) + 0.5
    gz, gy, gx = torch.meshgrid(r16, r16, r16, indexing="ij")
    d1 = cl[:, 0, None, None, None] + gx[None] - m3[:, 0, None, None, None]
    d2 = cl[:, 1, None, None, None] + gy[None] - m3[:, 1, None, None, None]
    d3 = cl[:, 2, None, None, None] + gz[None] - m3[:, 2, None, None, None]
    kk = [k[:, i, None, None, None] for i in range(6)]
    sig = (0.5 * (kk[0] * d1 * d1 + kk[3] * d2 * d2 + kk[5] * d3 * d3) + kk[1] * d1 * d2
           + kk[2] * d1 * d3 + kk[4] * d2 * d3)
    cut = torch.log(v["opacity"].to(f8) * 1e6)[:, None, None, None]
    near = (sig - cut).abs().reshape(C, -1).argmin(1)
    v_vol = torch.zeros((G, G, G), device=dev)
    v_vol[cl[:, 2] + near // 256, cl[:, 1] + (near // 16) % 16, cl[:, 0] + near % 16] = 1.0

    params = [t.clone().requires_grad_(True) for t in (means, quats, scales, opac)]
    st = E.prepare_explicit_gaussians(params[1], params[2], params[3], scale_min=wl.SCALE_MIN,
                                      scale_max=wl.SCALE_MAX)
    E.explicit_rasterize(st, params[0], torch.zeros((0, 4, 4), device=dev),
                         torch.zeros((0, 3, 3), device=dev), img_w=16, img_h=16,
                         tile_size=wl.IMG_TILE, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                         absgrad=False)
    vres = E.explicit_voxelize(st, params[0], rng, ctr, dim2=G, dim1=G, dim0=G,
                               tile_size=wl.VOL_TILE, eps3d=wl.EPS3D, radius_clip=clip)
    assert torch.equal(vres.radii, v["radii"])
    vres.volume.grad = v_vol
    E.explicit_backward(st, *params)
    theirs = ref.explicit_backward(None, None, v, v_vol, means, quats, scales, opac, covars, op,
                                   wl.SCALE_MIN, wl.SCALE_MAX)
    ref_keep = theirs["opacities"] != 0
    our_keep = params[3].grad != 0
    kept = int(ref_keep.sum())
    assert 0 < kept < C, kept
    assert torch.equal(our_keep, ref_keep), (
        f"{int((our_keep != ref_keep).sum())} of {C} voxel cut-off decisions differ")
    e = rel_l2(params[3].grad[ref_keep], theirs["opacities"][ref_keep])
    assert e < REL_L2_F32, e
