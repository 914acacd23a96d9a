"""The C-ABI library loads on a CPU-only machine and exports exactly what
include/r2s.h declares; argument errors are reported through status codes
and r2s_last_error without touching CUDA."""
import ctypes
import os
import re
import subprocess

import pytest

from _helpers import ROOT

HEADER = os.path.join(ROOT, "include", "r2s.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"R2S_API\s+[\w\s\*]+?\b(r2s_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from r2splat.cuda._backend import library_path, load_library

    path = library_path()
    if not os.path.exists(path):
        import importlib.util

        spec = importlib.util.spec_from_file_location(
            "r2s_build", os.path.join(ROOT, "bt-3dgs_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return load_library(path)


def test_header_declares_the_reference_operators():
    names = declared_functions()
    for op in ("parameter_transform_fwd", "parameter_transform_bwd", "isect_tiles_prepare",
               "isect_tiles_3d_prepare", "isect_offset_encode", "conics_mu_fwd", "conics_mu_bwd",
               "world_to_image_projection_fwd", "world_to_image_projection_bwd",
               "world_to_volume_mapping_fwd", "world_to_volume_mapping_bwd",
               "rasterize_to_pixels_fwd", "rasterize_to_pixels_bwd", "voxelize_to_voxels_fwd",
               "voxelize_to_voxels_bwd"):
        assert f"r2s_{op}" in names


def test_library_exports_every_declared_symbol(lib):
    from r2splat.cuda._backend import library_path

    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from {library_path()}"
    out = subprocess.run(["nm", "-D", "--defined-only", library_path()], capture_output=True,
                         text=True)
    if out.returncode == 0:
        exported = set(re.findall(r"\bT (r2s_\w+)", out.stdout))
        assert exported == set(declared_functions())


def test_ctypes_signatures_cover_the_header():
    from r2splat.cuda._backend import _SIGNATURES

    assert set(_SIGNATURES) == set(declared_functions())


def test_version_and_error_channel(lib):
    assert lib.r2s_version().startswith(b"r2s-b200")
    rc = lib.r2s_parameter_transform_fwd(0, None, None, 0.0, 1.0, None, None, -1, None)
    assert rc == 1  # R2S_ERR_ARG
    buf = ctypes.create_string_buffer(256)
    n = lib.r2s_last_error(buf, 256)
    assert n > 0 and b"negative" in buf.value
    # truncation keeps a terminated prefix
    small = ctypes.create_string_buffer(8)
    assert lib.r2s_last_error(small, 8) == n
    assert len(small.value) == 7


def test_invalid_arguments_are_rejected_before_any_launch(lib):
    # bad dtype code
    rc = lib.r2s_conics_mu_fwd(7, None, 0.0, None, None, 4, None)
    assert rc == 1
    # tile size beyond 32 (tile_size**2 > 1024)
    rc = lib.r2s_rasterize_to_pixels_fwd(0, None, None, None, None, None, None, 1, 1, 1, 64, 64, 33,
                                         2, 2, None, None, None)
    assert rc == 1
    buf = ctypes.create_string_buffer(256)
    lib.r2s_last_error(buf, 256)
    assert b"tile_size" in buf.value
    # non-positive radius clip
    rc = lib.r2s_world_to_image_projection_fwd(0, None, None, None, None, 1, 1, 8, 8, 0.0, 0.0, None,
                                               None, None, None)
    assert rc == 1


def test_workspace_sizes_are_bounded(lib):
    # config-2 shaped 2D binning: 75 views x 500k items x 1024 tiles
    b = lib.r2s_bin_workspace_bytes(75, 500_000, 1024, 0)
    assert 0 < b <= (256 << 20) + (1 << 20)
    # 3D: 32 layers of 32x32 bricks
    b3 = lib.r2s_bin_workspace_bytes(32, 500_000, 1024, 1)
    assert 0 < b3 <= (256 << 20) + (1 << 20)
    assert lib.r2s_bin_workspace_bytes(-1, 1, 1, 0) == -1


def test_training_entry_points_validate_arguments(lib):
    from r2splat.cuda._backend import AdamGroup

    buf = ctypes.create_string_buffer(256)
    groups = (AdamGroup * 9)()
    assert lib.r2s_adam_step_f32(groups, 9, 0.9, 0.999, 1e-15, None) == 1
    lib.r2s_last_error(buf, 256)
    assert b"groups" in buf.value
    one = (AdamGroup * 1)(AdamGroup(None, None, None, None, 4, 1e-3, 0))
    assert lib.r2s_adam_step_f32(one, 1, 0.9, 0.999, 1e-15, None) == 1  # step 0
    assert lib.r2s_adam_step_f32(one, 1, 1.5, 0.999, 1e-15, None) == 1  # beta out of range
    assert lib.r2s_densify_stats_f32(None, None, -1, 4, 1.0, 1.0, 1.0, None, None, None,
                                     None) == 1
    assert lib.r2s_densify_stats_f32(None, None, 1, 4, 1.0, 1.0, 0.0, None, None, None,
                                     None) == 1
    # the SSIM window of the reference configs is the only one built
    assert lib.r2s_projection_loss_f32(None, None, None, None, 1, 8, 8, 7, None, None, None,
                                       None, None) == 1
    lib.r2s_last_error(buf, 256)
    assert b"window" in buf.value
    assert lib.r2s_tv_loss_f32(None, 4, 4, 4, None, None, None, None) == 1
    assert lib.r2s_projection_loss_combine_f32(None, None, None, None, None, -1, None, None,
                                               None) == 1
