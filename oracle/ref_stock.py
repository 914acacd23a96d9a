"""The reference's own Python layers over the reference build -- TEST INFRASTRUCTURE ONLY.

``baseline/_ref`` holds the reference package as installed, unmodified, by
``python -m pip install --no-index --no-build-isolation --no-deps --target
baseline/_ref <reference checkout>`` with ``BUILD_NO_CUDA=1`` (its setup.py
switch that skips the extension, setup.py:10,77-78): the stock ``r2splat``
op layer (r2splat/ops/direct.py, explicit.py, r2splat/cuda/_wrapper.py,
_backend.py) and the ``src`` tree with ``GaussianModel``
(src/models/gaussian_model.py).  The extension those layers import as
``r2splat.csrc`` (r2splat/cuda/_backend.py:22) is the reference's CUDA
sources compiled for sm_100a by ``oracle/build_ref.py``
(``oracle/_ref/r2splat_ref_csrc.so``); it is registered under that name here.

This repository's package is also called ``r2splat``.  So the stock package
is loaded under the top-level alias ``ref_r2splat``: its relative imports
(including the lazy ``from ..cuda._wrapper import ...`` inside its op
functions) resolve inside the alias, and both packages live in one process.
``load_gaussian_model`` executes the unchanged gaussian_model.py with its
``from r2splat.ops ... import`` lines bound either to the stock package or to
this repository's, and ``src.utils.math`` taken from the same install, so the
same model class runs over either backend.  ``src/utils/__init__.py`` (which
pulls in matplotlib through validate.py) is not executed: ``src`` and
``src.utils`` are bare namespace stand-ins during that import.

Nothing in the product imports this module.
"""
from __future__ import annotations

import contextlib
import importlib
import importlib.util
import os
import sys
import types
from types import SimpleNamespace

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_PY = os.path.join(ROOT, "baseline", "_ref")
STOCK_ALIAS = "ref_r2splat"

_cache: dict = {}


def stock_available() -> bool:
    from oracle.ref_harness import reference_available

    return (os.path.isfile(os.path.join(REF_PY, "r2splat", "ops", "explicit.py"))
            and os.path.isfile(os.path.join(REF_PY, "src", "models", "gaussian_model.py"))
            and reference_available())


def _require():
    if not stock_available():
        raise FileNotFoundError(
            "stock reference layers missing: install the reference into baseline/_ref "
            "(BUILD_NO_CUDA=1 pip install --no-deps --target baseline/_ref <checkout>) and build "
            "oracle/_ref (python oracle/build_ref.py)")


def _load_package(alias: str, path: str):
    spec = importlib.util.spec_from_file_location(
        alias, os.path.join(path, "__init__.py"), submodule_search_locations=[path])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[alias] = mod
    spec.loader.exec_module(mod)
    return mod


def _load_file(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def stock_r2splat() -> SimpleNamespace:
    """The unchanged reference ``r2splat`` package (alias ``ref_r2splat``)
    over the reference build.  Returns its ``ops``, ``direct``, ``explicit``
    and ``wrapper`` modules."""
    if "stock" in _cache:
        return _cache["stock"]
    _require()
    from oracle.ref_harness import load_reference_module

    # r2splat/cuda/_backend.py:22 imports the extension by this absolute name
    sys.modules.setdefault("r2splat.csrc", load_reference_module())
    pkg = _load_package(STOCK_ALIAS, os.path.join(REF_PY, "r2splat"))
    ns = SimpleNamespace(
        package=pkg,
        ops=importlib.import_module(STOCK_ALIAS + ".ops"),
        direct=importlib.import_module(STOCK_ALIAS + ".ops.direct"),
        explicit=importlib.import_module(STOCK_ALIAS + ".ops.explicit"),
        wrapper=importlib.import_module(STOCK_ALIAS + ".cuda._wrapper"),
    )
    _cache["stock"] = ns
    return ns


@contextlib.contextmanager
def _bound_modules(bindings: dict):
    """Temporarily point sys.modules names at the given modules."""
    saved = {k: sys.modules.get(k) for k in bindings}
    try:
        sys.modules.update(bindings)
        yield
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def _src_math():
    if "src_math" not in _cache:
        _cache["src_math"] = _load_file("ref_src_utils_math",
                                        os.path.join(REF_PY, "src", "utils", "math.py"))
    return _cache["src_math"]


def _src_stubs(extra: dict | None = None) -> dict:
    src = types.ModuleType("src")
    src.__path__ = []
    utils = types.ModuleType("src.utils")
    utils.__path__ = []
    binds = {"src": src, "src.utils": utils, "src.utils.math": _src_math()}
    binds.update(extra or {})
    return binds


def load_gaussian_model(backend: str):
    """The reference's unchanged ``gaussian_model`` module
    (src/models/gaussian_model.py) with ``r2splat`` bound to ``backend``:
    ``"stock"`` (the reference op layer over the reference build) or
    ``"ours"`` (this repository's ``r2splat``)."""
    key = "gm_" + backend
    if key in _cache:
        return _cache[key]
    _require()
    if backend == "stock":
        s = stock_r2splat()
        r2 = {"r2splat": s.package, "r2splat.ops": s.ops, "r2splat.ops.direct": s.direct,
              "r2splat.ops.explicit": s.explicit}
    elif backend == "ours":
        ours = importlib.import_module("r2splat")
        import r2splat.ops as o_ops
        import r2splat.ops.direct as o_direct
        import r2splat.ops.explicit as o_explicit

        if os.path.commonpath([os.path.abspath(o_ops.__file__), REF_PY]) == REF_PY:
            raise RuntimeError("this repository's r2splat must come first on sys.path")
        r2 = {"r2splat": ours, "r2splat.ops": o_ops, "r2splat.ops.direct": o_direct,
              "r2splat.ops.explicit": o_explicit}
    else:
        raise ValueError(backend)
    with _bound_modules(_src_stubs(r2)):
        mod = _load_file(f"ref_gaussian_model_{backend}",
                         os.path.join(REF_PY, "src", "models", "gaussian_model.py"))
    _cache[key] = mod
    return mod


def load_binary_tree_model(backend: str):
    """``BinaryTreeGaussianModel`` (src/models/binary_tree_gaussian_model.py),
    unchanged, subclassing the ``GaussianModel`` of ``load_gaussian_model``."""
    key = "btm_" + backend
    if key in _cache:
        return _cache[key]
    gm = load_gaussian_model(backend)
    models = types.ModuleType("src.models")
    models.__path__ = []
    binds = _src_stubs({"src.models": models, "src.models.gaussian_model": gm})
    name = f"ref_binary_tree_model_{backend}"
    with _bound_modules(binds):
        # its relative import (.gaussian_model) resolves against __package__
        spec = importlib.util.spec_from_file_location(
            name, os.path.join(REF_PY, "src", "models", "binary_tree_gaussian_model.py"))
        mod = importlib.util.module_from_spec(spec)
        mod.__package__ = "src.models"
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    _cache[key] = mod
    return mod


def load_loss_module():
    """The reference's training losses (src/utils/loss.py, unchanged:
    ``BinaryTreeLossComputer``, ``LossComputer``, ``compute_tv_loss``) with
    ``src.utils.math`` and ``src.utils.metric`` from the same install."""
    if "loss" in _cache:
        return _cache["loss"]
    if "metric" not in _cache:
        _cache["metric"] = _load_file("ref_src_utils_metric",
                                      os.path.join(REF_PY, "src", "utils", "metric.py"))
    with _bound_modules(_src_stubs({"src.utils.metric": _cache["metric"]})):
        mod = _load_file("ref_src_utils_loss", os.path.join(REF_PY, "src", "utils", "loss.py"))
    _cache["loss"] = mod
    return mod


def load_strategy_module(backend: str = "stock"):
    """The reference's binary-tree strategy module
    (src/strategies/binary_tree.py, unchanged: ``split``, ``duplicate``,
    ``remove``, ``_append_history``, ``BinaryTreeStrategy``) with its imports
    (src/strategies/base.py, src/utils/ops.py, src/utils/math.py and the
    ``GaussianModel`` of ``load_gaussian_model(backend)``) from the same
    install."""
    key = "strategy_" + backend
    if key in _cache:
        return _cache[key]
    gm = load_gaussian_model(backend)
    models = types.ModuleType("src.models")
    models.__path__ = []
    strategies = types.ModuleType("src.strategies")
    strategies.__path__ = []
    binds = _src_stubs({"src.models": models, "src.models.gaussian_model": gm,
                        "src.strategies": strategies})
    with _bound_modules(binds):
        ops = _load_file("src.utils.ops", os.path.join(REF_PY, "src", "utils", "ops.py"))
        base = _load_file("src.strategies.base",
                          os.path.join(REF_PY, "src", "strategies", "base.py"))
        with _bound_modules({"src.utils.ops": ops, "src.strategies.base": base}):
            mod = _load_file("src.strategies.binary_tree",
                             os.path.join(REF_PY, "src", "strategies", "binary_tree.py"))
    # the modules stay reachable from the returned module's globals only
    for name in ("src.utils.ops", "src.strategies.base", "src.strategies.binary_tree"):
        sys.modules.pop(name, None)
    _cache[key] = mod
    return mod


__all__ = ["REF_PY", "stock_available", "stock_r2splat", "load_gaussian_model",
           "load_binary_tree_model", "load_loss_module", "load_strategy_module"]
