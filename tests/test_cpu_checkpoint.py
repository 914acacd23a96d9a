"""Checkpoint and export formats (r2s_checkpoint) against files written by the
reference's own serialisation methods (tests/golden/ckpt/, made by
tests/golden/make_checkpoint_fixtures.py from src/models/gaussian_model.py).
"""
import os
import pickle

import numpy as np
import pytest
import torch

import r2s_checkpoint as ck

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ckpt")
CASES = {"scalar": (7, ck.ScaleBound(5e-4, 1.0, 1e-4)),
         "axis": (5, ck.ScaleBound(np.array([1e-4, 2e-4, 3e-4], np.float32),
                                   np.array([0.5, 0.6, 0.7], np.float32), 2e-4)),
         "exp": (4, None)}


@pytest.fixture(scope="module")
def params():
    return torch.load(os.path.join(GOLD, "params.pt"), weights_only=True)


@pytest.mark.parametrize("name", sorted(CASES))
def test_load_reference_checkpoint(params, name):
    got, step = ck.load_ckpt(os.path.join(GOLD, f"{name}.ckpt"), strict=False)
    assert step == 100 + CASES[name][0]
    for k in ck.PARAM_NAMES:
        assert got[k].dtype == torch.float32 and torch.equal(got[k], params[name][k])


@pytest.mark.parametrize("name", sorted(CASES))
def test_saved_checkpoint_loads_like_the_reference(tmp_path, params, name):
    path = str(tmp_path / "m.ckpt")
    ck.save_ckpt(path, 7, params[name], extra={"note": name})
    payload = torch.load(path, weights_only=True)
    ref = torch.load(os.path.join(GOLD, f"{name}.ckpt"), weights_only=True)
    assert list(payload) == list(ref)  # step, model, extra keys in the same order
    assert list(payload["model"]) == list(ref["model"]) == list(ck.PARAM_NAMES)
    # the reference's load_ckpt: load_state_dict(strict=True) on the model's Parameters
    m = torch.nn.Module()
    for k in ck.PARAM_NAMES:
        setattr(m, k, torch.nn.Parameter(torch.zeros_like(params[name][k])))
    m.load_state_dict(payload["model"], strict=True)
    for k in ck.PARAM_NAMES:
        assert torch.equal(getattr(m, k), params[name][k])
    assert payload["step"] == 7 and payload["note"] == name


def test_strict_checkpoint_rejects_unknown_keys(tmp_path, params):
    path = str(tmp_path / "bad.ckpt")
    model = dict(params["scalar"])
    model["extra_buffer"] = torch.zeros(1)
    torch.save({"step": 1, "model": model}, path)
    with pytest.raises(RuntimeError, match="unexpected keys"):
        ck.load_ckpt(path, strict=True)
    got, step = ck.load_ckpt(path, strict=False)
    assert step == 1 and set(got) == set(ck.PARAM_NAMES)


@pytest.mark.parametrize("name", sorted(CASES))
def test_pickle_ply_is_byte_identical(tmp_path, params, name):
    path = str(tmp_path / "sub" / "m.ply")
    ck.save_ply(path, params[name], CASES[name][1])
    with open(path, "rb") as f, open(os.path.join(GOLD, f"{name}.ply"), "rb") as g:
        assert f.read() == g.read()


@pytest.mark.parametrize("name", sorted(CASES))
def test_load_reference_pickle_ply(params, name):
    got, bound = ck.load_ply(os.path.join(GOLD, f"{name}.ply"))
    for k in ck.PARAM_NAMES:
        assert torch.equal(got[k], params[name][k])
    want = CASES[name][1]
    if want is None:
        assert bound is None
    else:
        assert np.array_equal(bound.as_array(), want.as_array()) and bound.scale_eps == want.scale_eps


def test_pickle_ply_aliases_and_errors(tmp_path, params):
    p = params["scalar"]
    alias = {"means": p["means"].numpy(), "scales": p["scales"].numpy(),
             "quats": p["quats"].numpy(), "opacities": p["opacities"].numpy()}
    path = str(tmp_path / "alias.ply")
    with open(path, "wb") as f:
        pickle.dump(alias, f)
    got, bound = ck.load_ply(path)  # no scale_bound key: exp scales
    assert bound is None and all(torch.equal(got[k], p[k]) for k in ck.PARAM_NAMES)

    def write(d):
        with open(path, "wb") as f:
            pickle.dump(d, f)
        return path

    with pytest.raises(ValueError, match="Missing required fields"):
        ck.load_ply(write({"xyz": alias["means"]}))
    with pytest.raises(ValueError, match="Invalid scale_bound shape"):
        ck.load_ply(write({**alias, "scale_bound": np.zeros(3)}))
    with pytest.raises(AssertionError, match="greater than"):
        ck.load_ply(write({**alias, "scale_bound": np.array([1.0, 0.5])}))
    with pytest.raises(AssertionError, match="scale_eps"):
        ck.load_ply(write({**alias, "scale_bound": np.array([0.1, 0.5]), "scale_eps": 0.5}))


@pytest.mark.parametrize("name", sorted(CASES))
def test_ascii_export_is_byte_identical(tmp_path, params, name):
    path = str(tmp_path / "e.ply")
    assert ck.export_ply(path, params[name]["means"], params[name]["opacities"]) == path
    with open(path) as f, open(os.path.join(GOLD, f"{name}_export.ply")) as g:
        assert f.read() == g.read()
    with pytest.raises(ValueError, match="Unsupported color_mode"):
        ck.export_ply(path, params[name]["means"], params[name]["opacities"], color_mode="rgb")
