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
  src/strategies/binary_tree.py:305-347, non-packed path) in one launch.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Iterable, List, Union

import torch

from ..cuda import _wrapper as W
from ..cuda._backend import AdamGroup

__all__ = ["adam_step", "update_densify_state"]

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
