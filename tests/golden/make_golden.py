"""Generate the golden known-answer fixtures under tests/golden/.

Runs only where the reference checkout exists (``oracle.REFERENCE_ROOT``).  It
loads the dense PyTorch reference functions of the reference's own CUDA test
suite -- ``_covars_from_quats_scales_reference``,
``_unpack_covariance_reference``, ``_raster_reference`` and
``_voxel_reference`` in tests/test_cuda_gaussian_ops.py:32-50, 86-92,
200-238 -- by compiling just those function definitions out of the file's
AST, evaluates them (and torch.autograd through them) on the known-answer
inputs of the same tests, and writes ``kat.pt``.  The inputs restate those
tests (lines cited per case); where a test draws random inputs on the GPU,
the CPU generator with the same seed is used instead (the known answer is
the dense formula's value, so any input works).

Usage: ``python tests/golden/make_golden.py [reference_root]``
"""
from __future__ import annotations

import ast
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import REFERENCE_ROOT  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
HELPERS = (
    "_covars_from_quats_scales_reference",
    "_unpack_covariance_reference",
    "_raster_reference",
    "_voxel_reference",
)


def load_reference_helpers(ref_root: str) -> dict:
    path = os.path.join(ref_root, "tests", "test_cuda_gaussian_ops.py")
    tree = ast.parse(open(path).read(), filename=path)
    fns = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in HELPERS]
    missing = set(HELPERS) - {f.name for f in fns}
    if missing:
        raise RuntimeError(f"reference helpers not found: {sorted(missing)}")
    mod = ast.Module(body=fns, type_ignores=[])
    ns = {"torch": torch}
    exec(compile(mod, path, "exec"), ns)
    return ns


def main(ref_root: str = REFERENCE_ROOT) -> str:
    h = load_reference_helpers(ref_root)
    out = {}

    # parameter transform (test_cuda_gaussian_ops.py:53-83)
    g = torch.Generator().manual_seed(19)
    quats = torch.randn(11, 4, generator=g) * 0.7
    raw_scales = torch.randn(11, 3, generator=g)
    v_covars = torch.randn(11, 6, generator=g)
    smin, smax = 0.0005, 1.0
    q = quats.clone().requires_grad_(True)
    s = raw_scales.clone().requires_grad_(True)
    scales = smin + (smax - smin) * torch.sigmoid(s)
    cov = h["_covars_from_quats_scales_reference"](q, scales)
    gq, gs = torch.autograd.grad((cov * v_covars).sum(), (q, s))
    out["param"] = dict(quats=quats, raw_scales=raw_scales, v_covars=v_covars, scale_min=smin,
                        scale_max=smax, covars=cov.detach(), max_scales=scales.detach().amax(-1),
                        v_quats=gq, v_raw_scales=gs)

    # conics/mu near the det3 threshold (:95-152), computed in float64
    conic_cases = []
    base = torch.tensor(
        [[[1e-2, 0.0, 0.0, 1e-2, 0.0, f] for f in (1e-6, 9e-6, 11e-6, 1e-4)],
         [[1e-2, 2e-3, 1e-5, 2e-2, -2e-5, f] for f in (1e-6, 4e-6, 6e-6, 1e-4)]],
        dtype=torch.float64)
    for eps in (0.0, 1e-8):
        for mu_only in (True, False):
            ref = base.clone().requires_grad_(True)
            covm = h["_unpack_covariance_reference"](ref, eps)
            c2 = covm[..., :2, :2]
            d2 = torch.linalg.det(c2)
            d3 = torch.linalg.det(covm)
            inv2 = torch.linalg.inv(c2)
            conics_ref = inv2[..., (0, 0, 1), (0, 1, 1)]
            mus_ref = (2.0 * torch.pi * d3 / d2).sqrt()
            v_conics = torch.zeros_like(conics_ref.detach())
            if not mu_only:
                v_conics = torch.linspace(-0.2, 0.3, conics_ref.numel(),
                                          dtype=torch.float64).reshape_as(conics_ref)
            v_mus = torch.linspace(0.5, 1.2, mus_ref.numel(), dtype=torch.float64).reshape_as(mus_ref)
            full = torch.autograd.grad((conics_ref * v_conics).sum() + (mus_ref * v_mus).sum(), ref)[0]
            # conic-only part, for the kernels' cut-off of the mu term at det3 <= 1e-9
            ref2 = base.clone().requires_grad_(True)
            covm2 = h["_unpack_covariance_reference"](ref2, eps)
            inv2b = torch.linalg.inv(covm2[..., :2, :2])
            conic_grad = torch.autograd.grad((inv2b[..., (0, 0, 1), (0, 1, 1)] * v_conics).sum(), ref2,
                                             allow_unused=True)[0]
            if conic_grad is None:
                conic_grad = torch.zeros_like(base)
            conic_cases.append(dict(eps=eps, mu_only=mu_only, covars=base.clone(),
                                    conics=conics_ref.detach(), mus=mus_ref.detach(),
                                    v_conics=v_conics, v_mus=v_mus, grad=full,
                                    grad_conic_only=conic_grad, det3=d3.detach()))
    out["conics_mu"] = conic_cases

    # non-positive det3 keeps only conic gradients (:155-183)
    npd = []
    for last in (0.0, -1e-6):
        cov = torch.tensor([[[1e-2, 2e-3, 0.0, 2e-2, 0.0, last]]], dtype=torch.float64)
        ref = cov.clone().requires_grad_(True)
        covm = h["_unpack_covariance_reference"](ref, 0.0)
        inv2 = torch.linalg.inv(covm[..., :2, :2])
        conics_ref = inv2[..., (0, 0, 1), (0, 1, 1)]
        grad = torch.autograd.grad(conics_ref.sum(), ref)[0]
        npd.append(dict(covars=cov, conics=conics_ref.detach(), grad=grad))
    out["conics_nonpositive"] = npd

    # raster 2-Gaussian tile (:241-309)
    means = torch.tensor([[[5.2, 6.1], [10.0, 9.3]]], requires_grad=True)
    conics = torch.tensor([[[0.18, 0.01, 0.15], [0.12, -0.015, 0.2]]], requires_grad=True)
    opacity = torch.tensor([[0.7, 0.4]], requires_grad=True)
    mus = torch.tensor([[1.2, 0.8]], requires_grad=True)
    img = h["_raster_reference"](means, conics, opacity, mus, 16, 16)
    weight = torch.linspace(0.1, 1.0, img.numel()).reshape_as(img)
    grads = torch.autograd.grad((img * weight).sum(), (means, conics, opacity, mus))
    out["raster"] = dict(means2d=means.detach(), conics=conics.detach(), opacity=opacity.detach(),
                         mus=mus.detach(), image=img.detach(), weight=weight,
                         v_means2d=grads[0], v_conics=grads[1], v_opacity=grads[2], v_mus=grads[3])

    # voxel 2-Gaussian brick (:312-380)
    m3 = torch.tensor([[2.5, 3.1, 4.0], [5.2, 4.6, 3.3]], requires_grad=True)
    c3 = torch.tensor([[0.3, 0.01, 0.0, 0.25, -0.01, 0.2], [0.22, 0.0, 0.01, 0.28, 0.0, 0.24]],
                      requires_grad=True)
    o3 = torch.tensor([0.8, 0.5], requires_grad=True)
    vol = h["_voxel_reference"](m3, c3, o3, 8, 8, 8)
    w3 = torch.linspace(0.1, 1.0, vol.numel()).reshape_as(vol)
    g3 = torch.autograd.grad((vol * w3).sum(), (m3, c3, o3))
    out["voxel"] = dict(means3d=m3.detach(), conics=c3.detach(), opacity=o3.detach(),
                        volume=vol.detach(), weight=w3, v_means3d=g3[0], v_conics=g3[1],
                        v_opacity=g3[2])

    dst = os.path.join(HERE, "kat.pt")
    torch.save(out, dst)
    return dst


if __name__ == "__main__":
    print(main(sys.argv[1] if len(sys.argv) > 1 else REFERENCE_ROOT))
