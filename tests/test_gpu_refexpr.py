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
    kept = int(ref_keep.sum())
    assert 0 < kept < C, kept  # both decisions occur among the tested pixels
    assert torch.equal(our_keep, ref_keep), (
        f"{int((our_keep != ref_keep).sum())} of {C} cut-off decisions differ")
    # the kept values: opacity * vis from each build's own exponential (this
    # build's pre-scaled exp2, the reference's __expf)
    e = rel_l2(mine[4].reshape(C)[ref_keep], theirs[4].reshape(C)[ref_keep])
    assert e < REL_L2_F32, e
