"""Generate the checkpoint-format fixtures under tests/golden/ckpt/.

Runs only where the reference checkout exists (``oracle.REFERENCE_ROOT``).
The reference's ``GaussianModel`` module does not import here (its training
dependencies are absent), so this script compiles just the serialisation
methods out of the class's AST -- ``save_ckpt``, ``save_ply``,
``export_ply``, ``_get_scale_bound``, ``activated_opacities`` and
``activate_opacity`` (src/models/gaussian_model.py:98-100, 249-251, 556-676,
717-725) -- binds them to a small ``torch.nn.Module`` holding the four raw
parameters and the scale-bound attributes, and writes what they produce for
three seeded models: scalar sigmoid bounds, per-axis bounds, and exp scales
(no bounds).

The binary-tree checkpoint fixture (``tree.ckpt``, tensors in ``tree.pt``) is
written by the reference's ``BinaryTreeGaussianModel.save_ckpt`` itself
(src/models/binary_tree_gaussian_model.py:207-229): the class is executed
unchanged from the reference install in ``baseline/_ref`` by
``oracle/ref_stock.py`` (no GPU needed to save).

Usage: ``python tests/golden/make_checkpoint_fixtures.py [reference_root]``
"""
from __future__ import annotations

import ast
import os
import pickle
import sys

import numpy as np
import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import REFERENCE_ROOT  # noqa: E402

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ckpt")
METHODS = ("save_ckpt", "save_ply", "export_ply", "_get_scale_bound", "activated_opacities",
           "activate_opacity")


def reference_methods(root: str):
    src_path = os.path.join(root, "src", "models", "gaussian_model.py")
    tree = ast.parse(open(src_path).read())
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "GaussianModel")
    funcs = [n for n in cls.body if isinstance(n, ast.FunctionDef) and n.name in METHODS]
    assert {f.name for f in funcs} == set(METHODS), [f.name for f in funcs]
    body = ast.ClassDef(name="RefSerial", bases=[], keywords=[], body=funcs, decorator_list=[])
    mod = ast.Module(body=[body], type_ignores=[])
    ast.fix_missing_locations(mod)
    ns = {"os": os, "np": np, "torch": torch, "F": F, "pickle": pickle, "Optional": object,
          "Dict": dict, "Any": object}
    exec(compile(mod, src_path, "exec"), ns)
    return ns["RefSerial"]


def make_model(RefSerial, n, seed, bound):
    g = torch.Generator().manual_seed(seed)

    class Model(torch.nn.Module, RefSerial):
        pass

    m = Model()
    m.means = torch.nn.Parameter(torch.rand(n, 3, generator=g) - 0.5)
    m.scales = torch.nn.Parameter(torch.randn(n, 3, generator=g))
    m.quats = torch.nn.Parameter(torch.randn(n, 4, generator=g))
    m.opacities = torch.nn.Parameter(torch.randn(n, generator=g))
    if bound is None:
        m._use_sigmoid_scale = False
        m._scale_min = m._scale_max = None
        m._scale_eps = 0.0
    else:
        m._use_sigmoid_scale = True
        m._scale_min = torch.as_tensor(bound[0], dtype=torch.float32)
        m._scale_max = torch.as_tensor(bound[1], dtype=torch.float32)
        m._scale_eps = float(bound[2])
    return m


def main(root: str) -> None:
    RefSerial = reference_methods(root)
    os.makedirs(HERE, exist_ok=True)
    cases = {
        "scalar": (7, 11, (5e-4, 1.0, 1e-4)),
        "axis": (5, 12, ([1e-4, 2e-4, 3e-4], [0.5, 0.6, 0.7], 2e-4)),
        "exp": (4, 13, None),
    }
    params = {}
    for name, (n, seed, bound) in cases.items():
        m = make_model(RefSerial, n, seed, bound)
        m.save_ckpt(os.path.join(HERE, f"{name}.ckpt"), step=100 + n, extra={"note": name})
        m.save_ply(os.path.join(HERE, f"{name}.ply"))
        m.export_ply(os.path.join(HERE, f"{name}_export.ply"))
        params[name] = {k: getattr(m, k).detach().clone() for k in ("means", "scales", "quats", "opacities")}
    torch.save(params, os.path.join(HERE, "params.pt"))
    write_tree_fixture()
    print("wrote", sorted(os.listdir(HERE)))


def write_tree_fixture() -> None:
    from oracle import ref_stock

    mod = ref_stock.load_binary_tree_model("stock")
    m = mod.BinaryTreeGaussianModel(device="cpu", min_scale=5e-4, max_scale=1.0, scale_eps=1e-5)
    g = torch.Generator().manual_seed(14)
    n, h = 6, 3
    m.means = torch.nn.Parameter(torch.rand(n, 3, generator=g) - 0.5)
    m.scales = torch.nn.Parameter(torch.randn(n, 3, generator=g))
    m.quats = torch.nn.Parameter(torch.randn(n, 4, generator=g))
    m.opacities = torch.nn.Parameter(torch.randn(n, generator=g))
    m.parent = torch.tensor([-1, -1, 0, 0, 1, 1], dtype=torch.int32)
    m.level = torch.tensor([0, 0, 1, 1, 1, 1], dtype=torch.int32)
    m.history_means = torch.rand(h, 3, generator=g) - 0.5
    m.history_scales = torch.randn(h, 3, generator=g)
    m.history_quats = torch.randn(h, 4, generator=g)
    m.history_opacities = torch.randn(h, generator=g)
    m.history_parent = torch.tensor([-1, 0, 0], dtype=torch.int32)
    m.history_level = torch.tensor([0, 1, 1], dtype=torch.int32)
    m.save_ckpt(os.path.join(HERE, "tree.ckpt"), step=321, extra={"note": "tree"})
    names = ("means", "scales", "quats", "opacities", "parent", "level", "history_means",
             "history_scales", "history_quats", "history_opacities", "history_parent",
             "history_level")
    torch.save({k: getattr(m, k).detach().clone() for k in names}, os.path.join(HERE, "tree.pt"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else REFERENCE_ROOT)
