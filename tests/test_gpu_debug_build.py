"""The GPU workloads through the bounds-checked build (libr2s_debug.so,
R2S_DEBUG): every checked index stays in bounds and the results equal the
release library's.

A child process loads the checked library (R2S_LIBRARY) and runs the fused
op layer at config-1 scale -- projection with absolute gradients, the whole
grid and a z-slab of voxelization, both backwards, a projection split into
view batches under a forced record limit -- and the reference-layout
rasterizer, binning and voxelizer wrappers; then it reads the kernels' flag
words (r2s_debug_flags).  The flags must be clear, images, volumes and
integer outputs identical to the release build's and gradients equal up to
the order of their float additions.  This is the checked run that stands in
for a sanitizer run of the suite.
"""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

from _helpers import REL_L2_F32, ROOT, rel_l2

pytestmark = pytest.mark.gpu


def run_workloads():
    """The workloads; returns a dict of results (CPU tensors) and the flags."""
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W
    from r2splat.cuda._backend import _C
    from r2splat.ops import explicit as E

    cfg = wl.CONFIGS[1]
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(cfg, n=20_000))
    vm, K = wl.make_cameras(8, 256, total=cfg.n_views)
    vm, K = vm.cuda(), K.cuda()
    rng, ctr = (t.cuda() for t in wl.unit_cube_box())
    G, det = 128, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    v_img = torch.randn((8, det, det), generator=g, device="cuda")
    v_vol = torch.randn((G, G, G), generator=g, device="cuda")
    out = {}

    def step(tag, layers=None, v_volume=v_vol, limit=None):
        params = [t.clone().requires_grad_(True) for t in (m, q, s, o)]
        saved = W.MAX_RECORDS_PER_BATCH
        if limit is not None:
            W.MAX_RECORDS_PER_BATCH = limit
        try:
            st = E.prepare_explicit_gaussians(params[1], params[2], params[3],
                                              scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
            r = E.explicit_rasterize(st, params[0], vm, K, img_w=det, img_h=det,
                                     tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                     radius_clip=wl.RADIUS_CLIP, absgrad=True)
        finally:
            W.MAX_RECORDS_PER_BATCH = saved
        v = E.explicit_voxelize(st, params[0], rng, ctr, dim2=G, dim1=G, dim0=G,
                                tile_size=wl.VOL_TILE, eps3d=wl.EPS3D, radius_clip=wl.RADIUS_CLIP,
                                z_layers=layers)
        r.image.grad = v_img
        v.volume.grad = v_volume
        E.explicit_backward(st, *params)
        out[tag + "/image"] = r.image.detach().cpu()
        out[tag + "/volume"] = v.volume.detach().cpu()
        out[tag + "/radii"] = r.radii.cpu()
        out[tag + "/batches"] = torch.tensor(len(st.projection.buffers.view_batches or [0]))
        for name, p in zip(("means", "quats", "scales", "opac"), params):
            out[f"{tag}/grad_{name}"] = p.grad.cpu()
        out[tag + "/absgrad"] = r.means2d.absgrad.cpu()
        return st.projection.buffers.flatten_ids.numel()

    n_isects = step("full")
    step("slab", layers=(3, 9), v_volume=v_vol[24:72].contiguous())
    step("batched", limit=n_isects // 3)  # two or three of the 8 views per batch
    # reference-layout wrappers: binning with keys, rasterizer fwd/bwd, voxelizer fwd/bwd
    cov, max_s = W.parameter_transform_fwd(q, s, wl.SCALE_MIN, wl.SCALE_MAX)
    m2, c2, radii = W.world_to_image_projection_fwd(m, cov, vm, K, det, det, wl.EPS2D,
                                                    wl.RADIUS_CLIP)
    con, mus = W.conics_mu_fwd(c2, wl.EPS2D)
    op = torch.nn.functional.softplus(o)[None].expand(8, -1).contiguous()
    _, ids, fids = W.isect_tiles(m2, radii, 16, 16, 16)
    offs = W.isect_offset_encode(ids, 8, 16, 16)
    out["wrap/ids"], out["wrap/fids"] = ids.cpu(), fids.cpu()
    out["wrap/image"] = W.rasterize_to_pixels_fwd(m2, con, op, mus, offs, fids, det, det,
                                                  16).cpu()
    for k, t in enumerate(W.rasterize_to_pixels_bwd_per_gaussian(m2, con, op, mus, offs, ids, fids,
                                                                 v_img, det, det, 16, True)):
        out[f"wrap/raster_grad{k}"] = t.cpu()
    m3, c3, r3 = W.world_to_volume_mapping_fwd(m, cov, max_s, rng, ctr, G, G, G, wl.EPS3D,
                                               wl.RADIUS_CLIP)
    _, ids3, fids3 = W.isect_tiles_3d(m3, r3, 8, 16, 16, 16)
    offs3 = W.isect_offset_encode_3d(ids3, 16, 16, 16)
    op3 = torch.nn.functional.softplus(o).contiguous()
    out["wrap/volume"] = W.voxelize_to_voxels_fwd(m3, c3, op3, offs3, fids3, G, G, G, 8).cpu()
    for k, t in enumerate(W.voxelize_to_voxels_bwd_per_gaussian(m3, c3, op3, offs3, ids3, fids3,
                                                                v_vol, G, G, G, 8)):
        out[f"wrap/voxel_grad{k}"] = t.cpu()
    torch.cuda.synchronize()
    flags = ctypes.c_uint32(0)
    assert _C.r2s_debug_flags(ctypes.byref(flags), 1) == 0
    out["flags"] = torch.tensor(int(flags.value))
    out["debug_build"] = torch.tensor(int(_C.r2s_debug_build()))
    return out


def _child(path):
    torch.save(run_workloads(), path)


def test_checked_build_runs_clean_and_matches_release(tmp_path):
    debug_lib = os.path.join(ROOT, "bt-3dgs_b200", "r2splat", "_lib", "libr2s_debug.so")
    assert os.path.exists(debug_lib), "bounds-checked build missing: build.py --debug"
    out_path = str(tmp_path / "checked.pt")
    env = dict(os.environ, R2S_LIBRARY=debug_lib)
    code = ("import sys; sys.path[:0] = [{!r}, {!r}, {!r}]; import test_gpu_debug_build as T; "
            "T._child({!r})").format(os.path.join(ROOT, "tests"),
                                     os.path.join(ROOT, "bt-3dgs_b200"), ROOT, out_path)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=900)
    assert res.returncode == 0, res.stderr[-3000:]
    checked = torch.load(out_path)
    assert int(checked["debug_build"]) == 1, "the child did not load the checked build"
    assert int(checked["flags"]) == 0, f"bounds checks failed: flags {int(checked['flags']):#x}"
    release = run_workloads()
    assert int(release["debug_build"]) == 0 and int(release["flags"]) == 0
    assert int(checked["batched/batches"]) > 1
    for key, val in release.items():
        if key in ("flags", "debug_build"):
            continue
        other = checked[key]
        if "grad" in key:
            e = rel_l2(other, val)
            assert e < REL_L2_F32, f"{key}: rel-L2 {e:.3e}"
        else:
            assert torch.equal(other, val), key
