"""Training-step rows that follow the rasterizer backward, as fused kernels.

Not part of the reference's ``r2splat`` package: the reference runs these
steps in PyTorch inside its trainer and strategy.  A trainer that wants the
fused versions calls them in place of the PyTorch code they restate; both
work on the same tensors, so optimizer state dicts and strategy state stay
interchangeable.

* ``adam_step(optimizers)`` -- every ``torch.optim.Adam`` of the model
  (``GaussianModel.build_optimizers``, src/models/gaussian_model.py:514-530)
  stepped in one launch, in place of ``for opt in optimizers.values():
  opt.step()`` (src/trainers/binary_tree.py:204-205).
* ``update_densify_state(state, info, ...)`` -- the strategy's per-step
  statistics (``BinaryTreeStrategy._update_state``,
  src/strategies/binary_tree.py:305-347, non-packed path) in one launch;
  ``DensifyAccumulator(state)`` passed to ``explicit_backward(...,
  densify=...)`` computes the same statistics inside the backward kernel.
* ``FusedBinaryTreeLossComputer`` / ``FusedLossComputer`` -- the trainers'
  losses (``BinaryTreeLossComputer``, src/utils/loss.py:125-172;
  ``LossComputer``, loss.py:72-109): L1, SSIM and edge terms of the
  projections in one kernel each way, volume TV in one.
* ``binary_split(model, optimizers, state, mask, trainable_param_keys,
  revised_opacity)`` -- the binary-tree strategy's split
  (``split``, src/strategies/binary_tree.py:92-149) with the children's
  parameters computed in one launch (``r2s_split_children_f32``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Union

import torch

from ..cuda import _wrapper as W
from ..cuda._backend import AdamGroup

__all__ = ["DensifyAccumulator", "FusedBinaryTreeLossComputer", "FusedLossComputer", "adam_step",
           "binary_split", "projection_losses", "tv_loss", "update_densify_state"]

_MAX_GROUPS = 8


def _optimizer_list(optimizers) -> List[torch.optim.Optimizer]:
    if isinstance(optimizers, dict):
        return list(optimizers.values())
    if isinstance(optimizers, torch.optim.Optimizer):
        return [optimizers]
    return list(optimizers)


def _check_adam_group(group: dict) -> None:
    unsupported = [k for k, bad in (("amsgrad", True), ("maximize", True), ("differentiable", True),
                                    ("capturable", True), ("fused", True))
                   if group.get(k) == bad]
    if group.get("weight_decay", 0) != 0:
        unsupported.append("weight_decay")
    if unsupported:
        raise ValueError(f"adam_step supports plain Adam only; unsupported options: {unsupported}")


@torch.no_grad()
def adam_step(optimizers: Union[Dict[str, torch.optim.Adam], Iterable[torch.optim.Adam],
                                torch.optim.Adam]) -> None:
    """One Adam step of every parameter with a gradient, with torch.optim.Adam's
    state layout (``step`` as a CPU float32 tensor, ``exp_avg``,
    ``exp_avg_sq``) and arithmetic.  Parameters must be contiguous float32
    CUDA tensors; parameters without ``.grad`` are skipped, as in torch."""
    batches: Dict[tuple, list] = {}
    for opt in _optimizer_list(optimizers):
        if not isinstance(opt, torch.optim.Adam):
            raise TypeError(f"adam_step expects torch.optim.Adam, got {type(opt).__name__}")
        for group in opt.param_groups:
            _check_adam_group(group)
            beta1, beta2 = group["betas"]
            lr = float(group["lr"])
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("adam_step does not support sparse gradients")
                for name, t in (("param", p), ("grad", p.grad)):
                    W._check_cuda(name, t)
                    if t.dtype != torch.float32:
                        raise RuntimeError(f"adam_step: {name} must be float32")
                state = opt.state[p]
                if len(state) == 0:
                    state["step"] = torch.tensor(0.0, dtype=torch.float32)
                    state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                state["step"] += 1
                key = (p.device, float(beta1), float(beta2), float(group["eps"]))
                batches.setdefault(key, []).append(
                    (p, p.grad, state["exp_avg"], state["exp_avg_sq"], lr, int(state["step"].item())))
    for (device, beta1, beta2, eps), items in batches.items():
        for k in range(0, len(items), _MAX_GROUPS):
            chunk = items[k:k + _MAX_GROUPS]
            arr = (AdamGroup * len(chunk))()
            for i, (p, g, m, v, lr, step) in enumerate(chunk):
                arr[i] = AdamGroup(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(),
                                   p.numel(), lr, step)
            W._call("r2s_adam_step_f32", arr, len(chunk), beta1, beta2, eps, W._stream(device))


@torch.no_grad()
def update_densify_state(state: dict, info: dict, *, absgrad: bool = True,
                         key_for_gradient: str = "means2d", track_radii: bool = False) -> None:
    """``BinaryTreeStrategy._update_state`` for unpacked renders: accumulates
    ``state["grad2d"]``, ``state["count"]`` (and ``state["radii"]`` when
    ``track_radii``, the strategy's refine_scale2d_stop_iter > 0) from
    ``info[key_for_gradient].absgrad`` (or ``.grad``) and ``info["radii"]``."""
    for key in ("width", "height", "n_cameras", "radii", key_for_gradient):
        if key not in info:
            raise AssertionError(f"{key} is required but missing.")
    src = info[key_for_gradient]
    grads = src.absgrad if absgrad else src.grad
    if grads is None:
        raise RuntimeError(f"info[{key_for_gradient!r}] has no {'absgrad' if absgrad else 'grad'}")
    W._check_cuda("grads", grads)
    if grads.dtype != torch.float32 or grads.dim() != 3 or grads.size(-1) != 2:
        raise RuntimeError("update_densify_state: gradients must be float32 [C, N, 2]")
    C, N = grads.shape[:2]
    radii = info["radii"]
    if radii.shape != (C, N):
        raise RuntimeError(f"update_densify_state: radii must be [C, N] = [{C}, {N}]")
    radii = radii.to(torch.int32).contiguous()
    dev = grads.device
    if state.get("grad2d") is None:
        state["grad2d"] = torch.zeros(N, device=dev)
    if state.get("count") is None:
        state["count"] = torch.zeros(N, device=dev)
    if track_radii and state.get("radii") is None:
        state["radii"] = torch.zeros(N, device=dev)
    for key in ("grad2d", "count") + (("radii",) if track_radii else ()):
        t = state[key]
        W._check_cuda(f"state[{key!r}]", t)
        if t.dtype != torch.float32 or t.numel() != N:
            raise RuntimeError(f"update_densify_state: state[{key!r}] must be float32 [{N}]")
    width, height, n_cam = float(info["width"]), float(info["height"]), float(info["n_cameras"])
    W._call("r2s_densify_stats_f32", W._ptr(grads), W._ptr(radii), C, N,
            width / 2.0 * n_cam, height / 2.0 * n_cam, max(width, height),
            W._ptr(state["grad2d"]), W._ptr(state["count"]),
            W._ptr(state["radii"]) if track_radii else None, W._stream(dev))


@dataclass
class DensifyAccumulator:
    """``BinaryTreeStrategy._update_state`` fused into the explicit backward.

    Pass as ``explicit_backward(..., densify=DensifyAccumulator(state))``:
    the backward kernel that turns the raster statistics into the per-view
    screen-space gradients also adds, for every view where the Gaussian's
    radius is positive, the norm of its (scaled) absgrad -- or grad with
    ``absgrad=False`` -- to ``state["grad2d"]``, one to ``state["count"]`` and,
    with ``track_radii``, the radius over max(width, height) to
    ``state["radii"]`` (src/strategies/binary_tree.py:305-347).  The result is
    bit-identical to :func:`update_densify_state` on the same render, without
    the second pass over the [C, N, 2] gradients.  ``n_cameras`` defaults to
    the render's views (the adapter's ``info["n_cameras"]``).  With
    ``store_screen_grads=False`` the backward also skips writing
    ``means2d.grad`` / ``.absgrad`` (left None), whose only consumer in the
    reference's training step is this statistic."""

    state: dict
    absgrad: bool = True
    track_radii: bool = False
    n_cameras: Optional[int] = None
    store_screen_grads: bool = True

    def launch_args(self, radii: torch.Tensor, width: int, height: int):
        """The (radii, scale_x, scale_y, extent, absgrad, grad2d, count,
        max_radii) tuple of the fused entry point; creates the state tensors
        on first use as the strategy does."""
        C, N = radii.shape[:2]
        dev = radii.device
        if radii.dtype != torch.int32 or radii.shape != (C, N, 2) or not radii.is_contiguous():
            raise RuntimeError("densify: radii must be contiguous int32 [C, N, 2]")
        st = self.state
        if st.get("grad2d") is None:
            st["grad2d"] = torch.zeros(N, device=dev)
        if st.get("count") is None:
            st["count"] = torch.zeros(N, device=dev)
        if self.track_radii and st.get("radii") is None:
            st["radii"] = torch.zeros(N, device=dev)
        for key in ("grad2d", "count") + (("radii",) if self.track_radii else ()):
            t = st[key]
            W._check_cuda(f"state[{key!r}]", t)
            if t.dtype != torch.float32 or t.numel() != N or not t.is_contiguous():
                raise RuntimeError(f"densify: state[{key!r}] must be contiguous float32 [{N}]")
        n_cam = float(C if self.n_cameras is None else self.n_cameras)
        return (radii, float(width) / 2.0 * n_cam, float(height) / 2.0 * n_cam,
                float(max(width, height)), self.absgrad, st["grad2d"], st["count"],
                st["radii"] if self.track_radii else None)


# ---------------------------------------------------------------------------
# losses (BinaryTreeLossComputer, src/utils/loss.py:125-172)
# ---------------------------------------------------------------------------
def _image_stack(t: torch.Tensor, name: str) -> torch.Tensor:
    """[C, A, B] or single-channel [C, A, B, 1] -> contiguous float32 [C, A, B]."""
    if t.dim() == 4:
        if t.size(-1) != 1:
            raise RuntimeError(f"{name}: fused losses take single-channel images")
        t = t[..., 0]
    if t.dim() != 3:
        raise RuntimeError(f"{name}: expected [C, H, W] or [C, H, W, 1], got {tuple(t.shape)}")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name}: expected float32")
    t = t.contiguous()
    W._check_cuda(name, t)
    return t


_WINDOW_1D = {}


def _window_1d(window_size: int = 11):
    """The 1-D float32 SSIM weights exactly as the reference builds them
    (src/utils/metric.py:14-18: a float32 tensor of exp(-(x - ws//2)^2 /
    (2 sigma^2)), sigma 1.5, divided by its float32 sum)."""
    import math

    w = _WINDOW_1D.get(window_size)
    if w is None:
        g = torch.tensor([math.exp(-((x - window_size // 2) ** 2) / float(2 * 1.5 ** 2))
                          for x in range(window_size)])
        g = g / g.sum()
        w = (ctypes.c_float * window_size)(*[float(v) for v in g.tolist()])
        _WINDOW_1D[window_size] = w
    return w


class _ProjectionLoss(torch.autograd.Function):
    """(l1, ssim, edge) means of one batch of projections; gradient w.r.t. the
    renders only (the targets are data).  The forward pass also stores the
    SSIM gradient map, so the backward is one elementwise launch."""

    @staticmethod
    def forward(ctx, renders, targets, edge_targets, edge_mask):
        C, H, Wd = renders.shape
        dev = renders.device
        sums = torch.zeros(3, dtype=torch.float64, device=dev)
        dssim = None
        if ctx.needs_input_grad[0]:
            dssim = torch.empty_like(renders)
            unit = torch.tensor([0.0, 1.0, 0.0], dtype=torch.float32, device=dev)
        W._call("r2s_projection_loss_f32", W._ptr(renders), W._ptr(targets),
                W._ptr(edge_targets), W._ptr(edge_mask), C, H, Wd, 11, _window_1d(),
                W._ptr(unit) if dssim is not None else None, W._ptr(dssim), W._ptr(sums),
                W._stream(dev))
        ctx.save_for_backward(renders, targets, edge_targets, edge_mask, dssim)
        means = (sums / max(1, renders.numel())).float()
        return means[0], means[1], means[2]

    @staticmethod
    def backward(ctx, g_l1, g_ssim, g_edge):
        renders, targets, edge_targets, edge_mask, dssim = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        dev = renders.device
        weights = torch.stack([g if g is not None else torch.zeros((), device=dev)
                               for g in (g_l1, g_ssim, g_edge)]).float().contiguous()
        grad = torch.empty_like(renders)
        W._call("r2s_projection_loss_combine_f32", W._ptr(renders), W._ptr(targets),
                W._ptr(edge_targets), W._ptr(edge_mask), W._ptr(dssim), renders.numel(),
                W._ptr(weights), W._ptr(grad), W._stream(dev))
        return grad, None, None, None


class _TVLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vol):
        D0, D1, D2 = vol.shape
        s = torch.zeros(1, dtype=torch.float64, device=vol.device)
        W._call("r2s_tv_loss_f32", W._ptr(vol), D0, D1, D2, None, None, W._ptr(s),
                W._stream(vol.device))
        denom = (D0 - 1) * D1 * D2 + D0 * (D1 - 1) * D2 + D0 * D1 * (D2 - 1)
        ctx.save_for_backward(vol)
        return (s[0] / max(1, denom)).float()

    @staticmethod
    def backward(ctx, g):
        (vol,) = ctx.saved_tensors
        D0, D1, D2 = vol.shape
        grad = torch.empty_like(vol)
        s = torch.zeros(1, dtype=torch.float64, device=vol.device)
        weight = g.reshape(1).float().contiguous()
        W._call("r2s_tv_loss_f32", W._ptr(vol), D0, D1, D2, W._ptr(weight), W._ptr(grad),
                W._ptr(s), W._stream(vol.device))
        return grad


def projection_losses(renders, targets, edge_mask=None, edge_targets=None):
    """(l1, ssim, edge) means as differentiable device scalars (11x11 SSIM
    window); renders/targets [C, H, W] or [C, H, W, 1] float32 CUDA."""
    r = _image_stack(renders, "renders")  # indexing and contiguous() keep the autograd edge
    t = _image_stack(targets.detach(), "targets")
    et = em = None
    if edge_mask is not None:
        et = t if edge_targets is None else _image_stack(edge_targets.detach(), "edge_targets")
        em = _image_stack(edge_mask.detach().to(torch.float32), "edge_mask")
    if r.shape != t.shape:
        raise RuntimeError("renders and targets must have the same shape")
    return _ProjectionLoss.apply(r, t, et, em)


def tv_loss(volume):
    """compute_tv_loss(volume, reduction="mean") (src/utils/loss.py:10-21)."""
    vol = volume
    if vol.dim() == 4 and vol.size(0) == 1:
        vol = vol[0]
    if vol.dim() != 3:
        raise AssertionError("tv_3d_loss expects 3D volume")
    if vol.dtype != torch.float32:
        raise RuntimeError("tv_loss: expected float32")
    vol = vol.contiguous()
    W._check_cuda("volume", vol)
    return _TVLoss.apply(vol)


class FusedBinaryTreeLossComputer:
    """Drop-in for the reference's BinaryTreeLossComputer: same constructor,
    same call signature, same output keys; the projection terms and the
    volume TV come from the fused kernels (one pass each way)."""

    def __init__(self, w_l1: float, w_ssim: float, w_tv: float, w_edge: float,
                 w_hierarchy: float = 0.0, ssim_window: int = 11):
        if ssim_window != 11:
            raise ValueError("the fused losses are built for the 11-pixel SSIM window")
        self.w_l1, self.w_ssim, self.w_tv = w_l1, w_ssim, w_tv
        self.w_edge, self.w_hierarchy, self.ssim_window = w_edge, w_hierarchy, ssim_window

    def __call__(self, renders, targets, edge_mask=None, volume_pred=None, hierarchy_loss=None,
                 edge_targets=None, edge_weight_override=None):
        out = {}
        l1, ssim_val, edge_loss = projection_losses(renders, targets, edge_mask, edge_targets)
        if edge_mask is None:
            edge_loss = torch.zeros((), device=renders.device)
        out["proj_l1"] = l1
        out["proj_ssim"] = 1.0 - ssim_val
        if self.w_tv > 0 and volume_pred is not None:
            try:
                tv = tv_loss(volume_pred.squeeze())
            except Exception:
                tv = torch.zeros((), device=renders.device)
        else:
            tv = torch.zeros((), device=renders.device)
        out["vol_tv"] = tv
        out["edge"] = edge_loss
        if hierarchy_loss is None:
            hierarchy_loss = torch.zeros((), device=renders.device)
        out["hierarchy"] = hierarchy_loss
        edge_weight = self.w_edge if edge_weight_override is None else float(edge_weight_override)
        out["edge_weight"] = torch.tensor(edge_weight, device=renders.device)
        out["total"] = (self.w_l1 * l1 + self.w_ssim * out["proj_ssim"] + self.w_tv * tv
                        + edge_weight * edge_loss + self.w_hierarchy * hierarchy_loss)
        return out


class FusedLossComputer:
    """Drop-in for the reference's LossComputer (src/utils/loss.py:72-109):
    weighted projection L1 + SSIM and volume TV, from the fused kernels."""

    def __init__(self, w_l1: float, w_ssim: float, w_tv: float, ssim_window: int = 11):
        if ssim_window != 11:
            raise ValueError("the fused losses are built for the 11-pixel SSIM window")
        self.w_l1, self.w_ssim, self.w_tv, self.ssim_window = w_l1, w_ssim, w_tv, ssim_window

    def __call__(self, renders, targets, volume_pred=None):
        out = {}
        l1, ssim_val, _ = projection_losses(renders, targets)
        out["proj_l1"] = l1
        out["proj_ssim"] = 1.0 - ssim_val
        if self.w_tv > 0 and volume_pred is not None:
            try:
                tv = tv_loss(volume_pred.squeeze())
            except Exception:
                tv = torch.zeros((), device=renders.device)
        else:
            tv = torch.zeros((), device=renders.device)
        out["vol_tv"] = tv
        out["total"] = self.w_l1 * l1 + self.w_ssim * out["proj_ssim"] + self.w_tv * tv
        return out


# ---------------------------------------------------------------------------
# binary-tree split (src/strategies/binary_tree.py:17-149)
# ---------------------------------------------------------------------------
_TREE_HISTORY = (("history_means", "means"), ("history_scales", "scales"),
                 ("history_quats", "quats"), ("history_opacities", "opacities"),
                 ("history_parent", "parent"), ("history_level", "level"))


def _scale_bounds(model, scale_min, scale_max, scale_eps):
    lo = getattr(model, "_scale_min", None) if scale_min is None else scale_min
    hi = getattr(model, "_scale_max", None) if scale_max is None else scale_max
    eps = getattr(model, "_scale_eps", None) if scale_eps is None else scale_eps
    if lo is None or hi is None or eps is None:
        raise ValueError("binary_split needs sigmoid scale bounds (scale_min, scale_max, scale_eps)")
    lo, hi = torch.as_tensor(lo), torch.as_tensor(hi)
    if lo.numel() != 1 or hi.numel() != 1:
        raise ValueError("binary_split supports scalar scale bounds only")
    return float(lo.reshape(())), float(hi.reshape(())), float(eps)


@torch.no_grad()
def binary_split(model, optimizers: Dict[str, torch.optim.Optimizer], state: dict,
                 mask: torch.Tensor, trainable_param_keys: List[str],
                 revised_opacity: bool = False, *, scale_min: Optional[float] = None,
                 scale_max: Optional[float] = None, scale_eps: Optional[float] = None) -> None:
    """Split every Gaussian of ``mask`` into two children along its longest
    axis, in place, with the effects of the reference's ``split``
    (src/strategies/binary_tree.py:92-149) on the same objects:

    * ``model`` (anything with the raw parameters ``means``, ``scales``,
      ``quats``, ``opacities`` and the binary-tree buffers ``parent``,
      ``level``, ``history_*`` as attributes, e.g. the reference's
      ``BinaryTreeGaussianModel``): the selected nodes are archived at the end
      of the history (``_append_history``, :17-56), the parameters become
      [unselected rows; the S children at mean + offset; the S children at
      mean - offset], the children's parent is the archived node and their
      level its level + 1;
    * ``optimizers``: every moment buffer of a parameter keeps its rows of the
      unselected Gaussians and gets zeros for the children; the state moves
      to the new parameter (``_update_param_with_optimizer``,
      src/utils/ops.py:62-102);
    * ``state``: every tensor becomes [unselected rows; selected rows twice].

    The children's values come from one kernel (``r2s_split_children_f32``,
    float32, scalar sigmoid scale bounds taken from the model's
    ``_scale_min`` / ``_scale_max`` / ``_scale_eps`` unless given)."""
    lo, hi, eps = _scale_bounds(model, scale_min, scale_max, scale_eps)
    means = model.means
    dev = means.device
    sel = torch.where(mask)[0]
    rest = torch.where(~mask)[0]
    S = int(sel.numel())
    raw = {name: getattr(model, name) for name in ("means", "scales", "quats", "opacities")}
    for name, t in raw.items():
        if t.dtype != torch.float32 or not t.is_cuda:
            raise RuntimeError(f"binary_split: {name} must be a float32 CUDA tensor")
    children = {"means": torch.empty((2 * S, 3), dtype=torch.float32, device=dev),
                "scales": torch.empty((2 * S, 3), dtype=torch.float32, device=dev),
                "quats": torch.empty((2 * S, 4), dtype=torch.float32, device=dev),
                "opacities": torch.empty((2 * S,), dtype=torch.float32, device=dev)}
    sel64 = sel.to(torch.int64).contiguous()
    with torch.cuda.device(dev):
        W._call("r2s_split_children_f32", W._ptr(raw["means"].detach().contiguous()),
                W._ptr(raw["scales"].detach().contiguous()),
                W._ptr(raw["quats"].detach().contiguous()),
                W._ptr(raw["opacities"].detach().contiguous()), W._ptr(sel64), S, lo, hi, eps,
                1 if revised_opacity else 0, W._ptr(children["means"]),
                W._ptr(children["scales"]), W._ptr(children["quats"]),
                W._ptr(children["opacities"]), W._stream(dev))

    # archive the selected nodes (their current values) at the end of the history
    start = model.history_parent.shape[0]
    hist_idx = torch.arange(start, start + S, device=dev, dtype=torch.int32)
    if S:
        for hist, cur in _TREE_HISTORY:
            setattr(model, hist, torch.cat([getattr(model, hist),
                                            getattr(model, cur).index_select(0, sel).detach().clone()],
                                           dim=0))
    split_level = model.level.index_select(0, sel) + 1
    model.parent = torch.cat([model.parent.index_select(0, rest), hist_idx.repeat(2)], dim=0)
    model.level = torch.cat([model.level.index_select(0, rest), split_level.repeat(2)], dim=0)

    for name in trainable_param_keys:
        old = getattr(model, name)
        child = children.get(name)
        if child is None:
            child = old[sel].repeat([2] + [1] * (old.dim() - 1))
        new = torch.nn.Parameter(torch.cat([old[rest], child.to(old.dtype)]),
                                 requires_grad=old.requires_grad)
        setattr(model, name, new)
        if name not in optimizers:
            continue
        opt = optimizers[name]
        for group in opt.param_groups:
            pstate = opt.state.pop(old, {})
            for key in list(pstate.keys()):
                if key != "step":
                    v = pstate[key]
                    pstate[key] = torch.cat([v[rest], torch.zeros((2 * S, *v.shape[1:]),
                                                                  device=dev, dtype=v.dtype)])
            group["params"] = [new]
            opt.state[new] = pstate
    for k, v in state.items():
        if isinstance(v, torch.Tensor):
            state[k] = torch.cat((v[rest], v[sel].repeat([2] + [1] * (v.dim() - 1))))
