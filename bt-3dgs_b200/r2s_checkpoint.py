"""Checkpoint and export formats of the Gaussian parameters.

The reference keeps its parameters as four raw (pre-activation) tensors of
``GaussianModel`` and serialises them in three formats
(src/models/gaussian_model.py:556-676):

* **checkpoint** (``save_ckpt`` / ``load_ckpt``, :556-581): ``torch.save`` of
  ``{"step": int, "model": state_dict, **extra}`` where the state dict holds
  ``means`` [N,3], ``scales`` [N,3] (raw), ``quats`` [N,4] and ``opacities``
  [N] (raw), float32, in that registration order (:182-185).  The
  binary-tree model (src/models/binary_tree_gaussian_model.py:37-44,
  207-259) adds eight buffers after the parameters in its state dict --
  ``parent`` and ``level`` [N] int32, ``history_means`` [H,3],
  ``history_scales`` [H,3], ``history_quats`` [H,4], ``history_opacities``
  [H], ``history_parent`` and ``history_level`` [H] int32 -- and the same
  tensors again under a top-level ``"history"`` key (``save_ckpt(...,
  tree=...)``, ``load_tree_ckpt``);
* **pickle ``.ply``** (``save_ply`` / ``load_ply``, :583-641): a pickled dict
  of numpy arrays ``xyz``, ``density`` [N,1], ``scale``, ``rotation``, plus
  ``scale_bound`` (``[min, max]`` or a [2,3] array, ``None`` for exp scales)
  and ``scale_eps`` when the scales are sigmoid-bounded; the loader also
  accepts the aliases ``means``/``scales``/``quats``/``opacities`` and a
  squeezed density, and raises ``ValueError`` on missing fields or a bad
  ``scale_bound`` shape and ``AssertionError`` on inverted bounds or an eps
  outside [0, 0.5) (:620-626, :708-710, :736-745);
* **ASCII PLY export** (``export_ply``, :643-676): vertices with the activated
  opacity normalised to [0, 255] as a grey colour.

These functions read and write the same bytes from the raw tensors that the
operators of this package take (``prepare_explicit_gaussians(quats, scales,
opacities, ...)`` and the means), so a model trained with the reference loads
here and the other way round.  They are host-side I/O: nothing here runs on
the GPU beyond the device copies of the loaded tensors.
"""
from __future__ import annotations

import os
import pickle
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Dict, Mapping, Optional, Tuple, Union

import numpy as np
import torch

PARAM_NAMES = ("means", "scales", "quats", "opacities")
# binary-tree buffers in registration order (binary_tree_gaussian_model.py:37-44)
TREE_NAMES = ("parent", "level", "history_means", "history_scales", "history_quats",
              "history_opacities", "history_parent", "history_level")
_TREE_INT32 = ("parent", "level", "history_parent", "history_level")
_PLY_KEYS = {"means": ("xyz", "means"), "scales": ("scale", "scales"),
             "quats": ("rotation", "quats"), "opacities": ("density", "opacities")}


@dataclass
class ScaleBound:
    """Sigmoid scale bounds (scalars or per-axis [3] arrays) and their eps."""

    scale_min: Union[float, np.ndarray]
    scale_max: Union[float, np.ndarray]
    scale_eps: float = 1e-4

    def as_array(self) -> np.ndarray:
        """``scale_bound`` as the reference stores it (gaussian_model.py:717-725)."""
        lo = np.asarray(self.scale_min, dtype=np.float32)
        hi = np.asarray(self.scale_max, dtype=np.float32)
        if lo.ndim == 0:
            return np.array([float(lo), float(hi)])
        return np.stack([lo, hi], axis=0)


def _check_params(params: Mapping[str, torch.Tensor]) -> None:
    missing = [k for k in PARAM_NAMES if k not in params]
    if missing:
        raise ValueError(f"missing Gaussian parameters: {missing}")


def _check_tree(tree: Mapping[str, torch.Tensor]) -> None:
    missing = [k for k in TREE_NAMES if k not in tree]
    if missing:
        raise ValueError(f"missing binary-tree buffers: {missing}")


def save_ckpt(path: str, step: int, params: Mapping[str, torch.Tensor],
              extra: Optional[Dict[str, Any]] = None,
              tree: Optional[Mapping[str, torch.Tensor]] = None) -> None:
    """``torch.save({"step", "model": state_dict, **extra})`` with the
    reference's state-dict keys and order (gaussian_model.py:556-567).

    With ``tree`` (the eight binary-tree buffers of TREE_NAMES), the layout
    of ``BinaryTreeGaussianModel.save_ckpt``
    (binary_tree_gaussian_model.py:207-229): the buffers follow the
    parameters in the state dict and are stored again under ``"history"``,
    before the extra entries."""
    _check_params(params)
    model = OrderedDict((k, params[k].detach()) for k in PARAM_NAMES)
    payload: Dict[str, Any] = {"step": step, "model": model}
    if tree is not None:
        _check_tree(tree)
        for k in TREE_NAMES:
            model[k] = tree[k].detach()
        payload["history"] = {k: tree[k] for k in TREE_NAMES}
    if extra:
        payload.update(extra)
    torch.save(payload, path)


def load_ckpt(path: str, device: Union[str, torch.device] = "cpu",
              strict: bool = True) -> Tuple[Dict[str, torch.Tensor], int]:
    """Parameters and step of a checkpoint (gaussian_model.py:569-581).

    ``strict`` requires exactly the keys of the model that wrote it, as
    ``load_state_dict(strict=True)`` does (``RuntimeError`` otherwise): the
    four parameters, plus the eight binary-tree buffers when the checkpoint
    has the binary-tree layout (a ``"history"`` entry).  The buffers
    themselves are returned by ``load_tree_ckpt``.  The step is -1 when
    absent."""
    ckpt = torch.load(path, map_location=device, weights_only=True)
    model = ckpt["model"]
    if strict:
        expected = set(PARAM_NAMES) | (set(TREE_NAMES) if "history" in ckpt else set())
        keys = set(model.keys())
        if keys != expected:
            missing = sorted(expected - keys)
            unexpected = sorted(keys - expected)
            raise RuntimeError(f"Error(s) in loading state_dict: missing keys {missing}, "
                               f"unexpected keys {unexpected}")
    params = {k: model[k] for k in PARAM_NAMES if k in model}
    return params, int(ckpt.get("step", -1))


def load_tree_ckpt(path: str, device: Union[str, torch.device] = "cpu"
                   ) -> Tuple[Dict[str, torch.Tensor], Dict[str, torch.Tensor], int]:
    """Parameters, binary-tree buffers and step of a binary-tree checkpoint,
    as ``BinaryTreeGaussianModel.load_ckpt`` restores them
    (binary_tree_gaussian_model.py:231-259): parameters from the state dict,
    buffers from ``"history"`` (``KeyError`` when the checkpoint has none)
    with parent/level ids cast to int32."""
    ckpt = torch.load(path, map_location=device, weights_only=True)
    state = ckpt["model"]
    params = {k: state[k].to(device) for k in PARAM_NAMES}
    h = ckpt["history"]
    tree = {k: (h[k].to(device, dtype=torch.int32) if k in _TREE_INT32 else h[k].to(device))
            for k in TREE_NAMES}
    return params, tree, int(ckpt.get("step", -1))


def save_ply(path: str, params: Mapping[str, torch.Tensor],
             scale_bound: Optional[ScaleBound] = None) -> None:
    """Pickle ``.ply`` of the raw parameters (gaussian_model.py:583-608).

    ``scale_bound=None`` marks exp-activated scales (``scale_bound`` stored as
    None, no ``scale_eps``), as the reference does for an unbounded model."""
    _check_params(params)
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    density = params["opacities"].detach().cpu().numpy()
    if density.ndim == 1:
        density = density[:, None]
    out = {
        "xyz": params["means"].detach().cpu().numpy(),
        "density": density,
        "scale": params["scales"].detach().cpu().numpy(),
        "rotation": params["quats"].detach().cpu().numpy(),
        "scale_bound": None if scale_bound is None else scale_bound.as_array(),
    }
    if scale_bound is not None:
        out["scale_eps"] = scale_bound.scale_eps
    with open(path, "wb") as f:
        pickle.dump(out, f, pickle.HIGHEST_PROTOCOL)


def load_ply(path: str, device: Union[str, torch.device] = "cpu"
             ) -> Tuple[Dict[str, torch.Tensor], Optional[ScaleBound]]:
    """Raw float32 parameters and the scale bounds of a pickle ``.ply``
    (gaussian_model.py:610-641, 727-745)."""
    with open(path, "rb") as f:
        data = pickle.load(f)
    found = {}
    for name, (key, alias) in _PLY_KEYS.items():
        v = data.get(key, data.get(alias))
        found[name] = v
    if any(v is None for v in found.values()):
        raise ValueError(f"Missing required fields. Found keys: {list(data.keys())}")
    density = found["opacities"]
    if density.ndim == 2 and density.shape[1] == 1:
        density = density.squeeze(1)
    found["opacities"] = density
    params = {k: torch.tensor(v, dtype=torch.float32, device=device) for k, v in found.items()}

    sb = data.get("scale_bound", None)
    eps = data.get("scale_eps", 1e-4)
    if sb is None:
        return params, None
    sb = np.asarray(sb)
    if sb.shape == (2,):
        bound = ScaleBound(float(sb[0]), float(sb[1]), float(eps))
    elif sb.shape == (2, 3):
        bound = ScaleBound(sb[0], sb[1], float(eps))
    else:
        raise ValueError(f"Invalid scale_bound shape: {sb.shape}")
    # the reference's _configure_scale_bounds asserts these (:708-710)
    lo = np.asarray(bound.scale_min, dtype=np.float32)
    hi = np.asarray(bound.scale_max, dtype=np.float32)
    if not np.all(hi > lo):
        raise AssertionError("max_scale must be greater than min_scale")
    if not 0.0 <= bound.scale_eps < 0.5:
        raise AssertionError("scale_eps must lie in [0, 0.5)")
    return params, bound


def export_ply(path: str, means: torch.Tensor, raw_opacities: torch.Tensor,
               color_mode: str = "opacity") -> str:
    """ASCII PLY of the means with the softplus-activated opacity, min-max
    normalised to [0, 255], as grey (gaussian_model.py:643-676)."""
    if color_mode not in ("opacity", "density"):
        raise ValueError(f"Unsupported color_mode: {color_mode}")
    pts = means.detach().cpu().numpy()
    post = torch.nn.functional.softplus(raw_opacities.detach()).cpu().numpy()
    vals = post.reshape(-1)
    vmin, vmax = float(vals.min()), float(vals.max())
    norm = (vals - vmin) if vmax - vmin < 1e-8 else (vals - vmin) / (vmax - vmin)
    colors = (norm * 255.0).clip(0, 255).astype("uint8")
    lines = ["ply\nformat ascii 1.0\n", f"element vertex {pts.shape[0]}\n",
             "property float x\nproperty float y\nproperty float z\n",
             "property uchar red\nproperty uchar green\nproperty uchar blue\n", "end_header\n"]
    lines += [f"{x} {y} {z} {c} {c} {c}\n" for (x, y, z), c in zip(pts, colors)]
    with open(path, "w") as f:
        f.write("".join(lines))
    return path
