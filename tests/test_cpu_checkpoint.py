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


@pytest.fixture(scope="module")
def tree():
    return torch.load(os.path.join(GOLD, "tree.pt"), weights_only=True)


def test_load_reference_binary_tree_checkpoint(tree):
    """tree.ckpt was written by BinaryTreeGaussianModel.save_ckpt: a strict
    load accepts its buffers, load_tree_ckpt returns them as the reference's
    load_ckpt restores them (binary_tree_gaussian_model.py:231-259)."""
    path = os.path.join(GOLD, "tree.ckpt")
    params, step = ck.load_ckpt(path, strict=True)
    assert step == 321 and list(params) == list(ck.PARAM_NAMES)
    p2, buffers, step2 = ck.load_tree_ckpt(path)
    assert step2 == 321
    for k in ck.PARAM_NAMES:
        assert torch.equal(params[k], tree[k]) and torch.equal(p2[k], tree[k])
    for k in ck.TREE_NAMES:
        assert torch.equal(buffers[k], tree[k]), k
        if k in ("parent", "level", "history_parent", "history_level"):
            assert buffers[k].dtype == torch.int32


def test_saved_binary_tree_checkpoint_matches_the_reference_layout(tmp_path, tree):
    path = str(tmp_path / "t.ckpt")
    ck.save_ckpt(path, 321, {k: tree[k] for k in ck.PARAM_NAMES},
                 extra={"note": "tree"}, tree={k: tree[k] for k in ck.TREE_NAMES})
    payload = torch.load(path, weights_only=True)
    ref = torch.load(os.path.join(GOLD, "tree.ckpt"), weights_only=True)
    assert list(payload) == list(ref)  # step, model, history, extra
    assert list(payload["model"]) == list(ref["model"])
    assert list(payload["history"]) == list(ref["history"])
    for k in ref["model"]:
        assert torch.equal(payload["model"][k], ref["model"][k])
        assert payload["model"][k].dtype == ref["model"][k].dtype
    for k in ref["history"]:
        assert torch.equal(payload["history"][k], ref["history"][k])
    assert payload["note"] == "tree"
    _, buffers, _ = ck.load_tree_ckpt(path)
    assert all(torch.equal(buffers[k], tree[k]) for k in ck.TREE_NAMES)


def test_binary_tree_checkpoint_errors(tmp_path, tree):
    with pytest.raises(ValueError, match="missing binary-tree buffers"):
        ck.save_ckpt(str(tmp_path / "x.ckpt"), 1, {k: tree[k] for k in ck.PARAM_NAMES},
                     tree={"parent": tree["parent"]})
    # a base-model checkpoint has no history: the tree loader fails like the reference's
    with pytest.raises(KeyError):
        ck.load_tree_ckpt(os.path.join(GOLD, "scalar.ckpt"))
    # tree buffers without the history entry are unexpected keys for a strict load
    path = str(tmp_path / "y.ckpt")
    model = {k: tree[k] for k in ck.PARAM_NAMES + ck.TREE_NAMES}
    torch.save({"step": 1, "model": model}, path)
    with pytest.raises(RuntimeError, match="unexpected keys"):
        ck.load_ckpt(path, strict=True)
