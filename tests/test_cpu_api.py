"""The Python drop-in surface on a machine without CUDA: import contract,
names and signatures of the reference API, and its error behaviour."""
import inspect
import os
import subprocess
import sys

import pytest
import torch

from _helpers import ROOT


def test_import_touches_no_cuda():
    """Same contract as the reference's tests/test_release_imports.py:9-34."""
    code = f"""
import sys
sys.path[:0] = [{os.path.join(ROOT, 'bt-3dgs_b200')!r}]
import torch
def forbidden(*a, **k):
    raise AssertionError('import touched CUDA')
torch.cuda.is_available = forbidden
torch.cuda.init = forbidden
import r2splat, r2splat.ops, r2splat.ops.direct, r2splat.ops.explicit, r2splat.cuda._wrapper
from r2splat.cuda._backend import _lazy_C
assert not _lazy_C._load_attempted
"""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                         timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr


def test_public_names_match_the_reference():
    import r2splat
    import r2splat.ops as ops
    import r2splat.ops.explicit as ex
    import r2splat.cuda._wrapper as W

    assert set(ops.__all__) == {
        "ExplicitGaussianState", "InferenceGaussianState", "MappingVoxelizationResult",
        "ProjectionRasterizationResult", "inference_rasterize", "inference_voxelize",
        "prepare_inference_gaussians"}
    assert set(ex.__all__) == {"ExplicitGaussianState", "explicit_backward", "explicit_rasterize",
                               "explicit_voxelize", "prepare_explicit_gaussians"}
    assert r2splat.InferenceGaussianState is ops.InferenceGaussianState
    ops18 = ["isect_tiles", "parameter_transform_fwd", "parameter_transform_bwd",
             "isect_offset_encode", "isect_tiles_3d", "isect_offset_encode_3d", "conics_mu_fwd",
             "conics_mu_bwd", "world_to_image_projection_fwd", "world_to_image_projection_bwd",
             "world_to_volume_mapping_fwd", "world_to_volume_mapping_bwd",
             "rasterize_to_pixels_fwd", "rasterize_to_pixels_bwd",
             "rasterize_to_pixels_bwd_per_gaussian", "voxelize_to_voxels_fwd",
             "voxelize_to_voxels_bwd", "voxelize_to_voxels_bwd_per_gaussian"]
    for name in ops18:
        assert callable(getattr(W, name))
    # positional arity of the reference bindings (include/Ops.h:9-79)
    arity = {"parameter_transform_fwd": 4, "parameter_transform_bwd": 5, "isect_tiles": 5,
             "isect_offset_encode": 4, "isect_tiles_3d": 6, "isect_offset_encode_3d": 4,
             "conics_mu_fwd": 2, "conics_mu_bwd": 6, "world_to_image_projection_fwd": 8,
             "world_to_image_projection_bwd": 8, "world_to_volume_mapping_fwd": 10,
             "world_to_volume_mapping_bwd": 10, "rasterize_to_pixels_fwd": 9,
             "rasterize_to_pixels_bwd": 11, "rasterize_to_pixels_bwd_per_gaussian": 12,
             "voxelize_to_voxels_fwd": 9, "voxelize_to_voxels_bwd": 10,
             "voxelize_to_voxels_bwd_per_gaussian": 11}
    for name, n in arity.items():
        assert len(inspect.signature(getattr(W, name)).parameters) == n, name


def test_keyword_only_arguments_of_the_op_layer():
    from r2splat.ops import direct, explicit

    sig = inspect.signature(direct.inference_rasterize)
    kw = [p.name for p in sig.parameters.values() if p.kind == p.KEYWORD_ONLY]
    assert kw == ["img_w", "img_h", "tile_size", "eps2d", "radius_clip"]
    sig = inspect.signature(explicit.explicit_rasterize)
    kw = [p.name for p in sig.parameters.values() if p.kind == p.KEYWORD_ONLY]
    assert kw == ["img_w", "img_h", "tile_size", "eps2d", "radius_clip", "absgrad"]
    sig = inspect.signature(direct.inference_voxelize)
    kw = [p.name for p in sig.parameters.values() if p.kind == p.KEYWORD_ONLY]
    assert kw == ["dim2", "dim1", "dim0", "tile_size", "eps3d", "radius_clip"]


def test_cpu_tensors_are_rejected_like_the_reference():
    from r2splat.ops import direct

    q = torch.zeros(2, 4)
    with pytest.raises(RuntimeError, match="require CUDA tensors"):
        direct.prepare_inference_gaussians(q, torch.zeros(2, 3), torch.zeros(2), scale_min=5e-4,
                                           scale_max=1.0)


def test_bad_tile_sizes_raise_value_error():
    from r2splat.ops import direct

    state = direct.InferenceGaussianState(torch.zeros(1, 6), torch.zeros(1), torch.zeros(1))
    with pytest.raises(ValueError, match="tile_size"):
        direct.inference_rasterize(state, torch.zeros(1, 3), torch.eye(4)[None], torch.eye(3)[None],
                                   img_w=8, img_h=8, tile_size=33, eps2d=1e-8, radius_clip=3.0)
    with pytest.raises(ValueError, match="tile_size"):
        direct.inference_voxelize(state, torch.zeros(1, 3), torch.ones(3), torch.zeros(3), dim2=8,
                                  dim1=8, dim0=8, tile_size=11, eps3d=1e-8, radius_clip=3.0)


def test_backward_mode_validation_and_single_use_state():
    from r2splat.ops import explicit

    with pytest.raises(ValueError, match="backward_mode"):
        explicit._validate_backward_mode("bogus")
    st = explicit.ExplicitGaussianState(torch.zeros(1, 6), torch.zeros(1), torch.zeros(1), 5e-4,
                                        1.0, "primitive")
    with pytest.raises(RuntimeError, match="projection forward pass"):
        explicit.explicit_backward(st, torch.zeros(1, 3), torch.zeros(1, 4), torch.zeros(1, 3),
                                   torch.zeros(1))
    st.projection = object()
    with pytest.raises(RuntimeError, match="rasterized once"):
        explicit.explicit_rasterize(st, torch.zeros(1, 3), torch.eye(4)[None], torch.eye(3)[None],
                                    img_w=8, img_h=8, tile_size=16, eps2d=1e-8, radius_clip=3.0,
                                    absgrad=False)
    st.voxel = object()
    with pytest.raises(RuntimeError, match="voxelized once"):
        explicit.explicit_voxelize(st, torch.zeros(1, 3), torch.ones(3), torch.zeros(3), dim2=8,
                                   dim1=8, dim0=8, tile_size=8, eps3d=1e-8, radius_clip=3.0)
    st.backward_called = True
    with pytest.raises(RuntimeError, match="only run once"):
        explicit.explicit_backward(st, torch.zeros(1, 3), torch.zeros(1, 4), torch.zeros(1, 3),
                                   torch.zeros(1))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_wrapper_without_cuda_raises_runtime_error():
    import r2splat.cuda._wrapper as W

    assert W.is_cuda_extension_available() is False
    with pytest.raises(RuntimeError):
        W.conics_mu_fwd(torch.zeros(1, 1, 6), 0.0)


def test_adam_step_rejects_unsupported_options():
    from r2splat.ops.training import adam_step

    p = torch.nn.Parameter(torch.zeros(3))
    p.grad = torch.zeros(3)
    for kwargs in ({"amsgrad": True}, {"weight_decay": 0.1}, {"maximize": True}):
        with pytest.raises(ValueError, match="unsupported"):
            adam_step(torch.optim.Adam([p], lr=0.1, **kwargs))
    with pytest.raises(TypeError):
        adam_step([torch.optim.SGD([p], lr=0.1)])
