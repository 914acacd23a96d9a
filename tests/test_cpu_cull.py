"""Conservativeness of the exact tile culling (csrc/r2s_cull.cuh) on the CPU.

The 16x16 rasterizer kernels narrow each record's culling box to the rows
(and columns) where its ellipse meets the tile.  Dropping a pixel that the
float32 cut-off test would count changes the image and the gradients, so
the harness in ``cull_probe.cpp`` re-evaluates every pixel of the starting
box in the kernels' own float32 operation orders and counts passing pixels
outside the narrowed ranges; there must be none.  Cases: realistic splats
(sizes 0.3-300 px, any orientation, signed amplitudes), tiny and huge
ellipses, conditioning up to 1e6, means on pixel centres and tile edges,
strips that graze the ellipse, partial tiles and random starting boxes.
"""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "bt-3dgs_b200", "csrc")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("cull") / "libcullprobe.so")
    subprocess.run([gxx, "-O2", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC", "-I", CSRC,
                    os.path.join(HERE, "cull_probe.cpp"), "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.cull_probe.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.cull_probe.restype = ctypes.c_int

    def run(cases, boxes):
        cases = np.ascontiguousarray(cases, dtype=np.float32)
        boxes = np.ascontiguousarray(boxes, dtype=np.int32)
        out = np.zeros((len(cases), 8), dtype=np.int32)
        lib.cull_probe(cases.ctypes.data, boxes.ctypes.data, len(cases), out.ctypes.data)
        return out

    return run


def _conics(rng, n, log_sig_lo, log_sig_hi, max_cond=None):
    s1 = np.exp(rng.uniform(log_sig_lo, log_sig_hi, n))
    if max_cond is None:
        s2 = np.exp(rng.uniform(log_sig_lo, log_sig_hi, n))
    else:  # eigenvalue ratio up to max_cond
        s2 = s1 / np.sqrt(np.exp(rng.uniform(0, np.log(max_cond), n)))
    th = rng.uniform(0, np.pi, n)
    ct, st = np.cos(th), np.sin(th)
    # conic = R diag(1/s1^2, 1/s2^2) R^T
    l1, l2 = 1 / s1**2, 1 / s2**2
    a = ct * ct * l1 + st * st * l2
    b = ct * st * (l1 - l2)
    c = st * st * l1 + ct * ct * l2
    return a, b, c, np.maximum(s1, s2)


def _cases(rng, n, log_sig_lo, log_sig_hi, max_cond=None, snap=False):
    a, b, c, smax = _conics(rng, n, log_sig_lo, log_sig_hi, max_cond)
    wmu = np.exp(rng.uniform(np.log(1e-5), np.log(20.0), n)) * rng.choice([-1.0, 1.0], n)
    X0 = 16.0 * rng.integers(0, 64, n)
    Y0 = 16.0 * rng.integers(0, 64, n)
    reach = 8.0 + np.minimum(4.0 * smax, 4000.0)
    mx = X0 + 8.0 + rng.uniform(-1, 1, n) * reach
    my = Y0 + 8.0 + rng.uniform(-1, 1, n) * reach
    if snap:  # means on pixel centres / tile edges
        mx = np.floor(mx) + rng.choice([0.0, 0.5], n)
        my = np.floor(my) + rng.choice([0.0, 0.5], n)
    return np.stack([mx, my, a, b, c, wmu, X0, Y0], -1).astype(np.float32)


def _boxes(rng, n, random_box):
    cmax = np.where(rng.random(n) < 0.2, rng.integers(0, 16, n), 15)
    rmax = np.where(rng.random(n) < 0.2, rng.integers(0, 16, n), 15)
    if random_box:
        c0 = rng.integers(0, 16, n)
        c1 = np.minimum(c0 + rng.integers(0, 16, n), cmax)
        r0 = rng.integers(0, 16, n)
        r1 = np.minimum(r0 + rng.integers(0, 16, n), rmax)
    else:
        c0, c1, r0, r1 = np.zeros(n, int), cmax, np.zeros(n, int), rmax
    return np.stack([c0, c1, r0, r1, cmax, rmax], -1).astype(np.int32)


@pytest.mark.parametrize("kind", ["realistic", "tiny", "huge", "ill_conditioned", "snapped",
                                  "random_boxes"])
def test_tile_cull_never_drops_a_passing_pixel(probe, kind):
    rng = np.random.default_rng(["realistic", "tiny", "huge", "ill_conditioned", "snapped",
                                 "random_boxes"].index(kind) + 11)
    n = 40000
    if kind == "realistic":
        cases = _cases(rng, n, np.log(0.3), np.log(300.0))
    elif kind == "tiny":
        cases = _cases(rng, n, np.log(0.02), np.log(0.5))
    elif kind == "huge":
        cases = _cases(rng, n, np.log(100.0), np.log(3000.0))
    elif kind == "ill_conditioned":
        cases = _cases(rng, n, np.log(0.5), np.log(200.0), max_cond=1e6)
    else:
        cases = _cases(rng, n, np.log(0.3), np.log(100.0), snap=kind == "snapped")
    out = probe(cases, _boxes(rng, n, kind == "random_boxes"))
    bad = np.nonzero(out[:, 4])[0]
    assert len(bad) == 0, f"{len(bad)} cases drop passing pixels, first: {cases[bad[0]]} -> {out[bad[0]]}"


def test_tile_cull_is_tight_on_tilted_splats(probe):
    """On realistic tilted splats the narrowed ranges stay close to the rows
    and columns that actually hold passing pixels."""
    rng = np.random.default_rng(5)
    n = 40000
    cases = _cases(rng, n, np.log(1.0), np.log(30.0))
    out = probe(cases, _boxes(rng, n, False))
    live = out[:, 7] > 0
    nrows = np.maximum(out[:, 3] - out[:, 2] + 1, 0)
    ncols = np.maximum(out[:, 1] - out[:, 0] + 1, 0)
    assert (nrows[live] >= out[live, 5]).all() and (ncols[live] >= out[live, 6]).all()
    # at most one spare row/column per side on average, few records kept without a pixel
    assert nrows[live].mean() <= out[live, 5].mean() + 1.0
    assert ncols[live].mean() <= out[live, 6].mean() + 1.0
    assert (nrows[~live] > 0).mean() < 0.2


def test_tile_cull_keeps_degenerate_records(probe):
    """Degenerate conics, non-finite values and sub-threshold amplitudes
    keep their box (the per-pixel test decides)."""
    rows = [
        [8.0, 8.0, 1.0, 2.0, 1.0, 1.0, 0.0, 0.0],  # det < 0
        [8.0, 8.0, 0.0, 0.0, 1.0, 1.0, 0.0, 0.0],  # a = 0
        [np.nan, 8.0, 1.0, 0.0, 1.0, 1.0, 0.0, 0.0],
        [8.0, 8.0, 1.0, 0.0, 1.0, np.nan, 0.0, 0.0],
        [8.0, 8.0, 1.0, 0.0, 1.0, np.inf, 0.0, 0.0],
        [8.0, 8.0, 1.0, 0.0, 1.0, 1e-7, 0.0, 0.0],  # below the cut-off: no pixel passes
    ]
    cases = np.array(rows, dtype=np.float32)
    boxes = np.tile(np.array([[0, 15, 0, 15, 15, 15]], dtype=np.int32), (len(rows), 1))
    out = probe(cases, boxes)
    for k in range(len(rows)):
        assert out[k, 4] == 0
        assert tuple(out[k, :4]) == (0, 15, 0, 15), (rows[k], out[k])


def _rotations(rng, n):
    q = rng.standard_normal((n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    return np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)], -2)


def _cases3(rng, n, lo, hi, max_cond=None, snap=False):
    s = np.exp(rng.uniform(np.log(lo), np.log(hi), (n, 3)))
    if max_cond is not None:
        s[:, 2] = s[:, 0] / np.sqrt(np.exp(rng.uniform(0, np.log(max_cond), n)))
    R = _rotations(rng, n)
    P = R @ (np.eye(3)[None] / (s * s)[:, None, :]) @ R.transpose(0, 2, 1)  # conic = R S^-2 R^T
    q = np.stack([P[:, 0, 0], P[:, 0, 1], P[:, 0, 2], P[:, 1, 1], P[:, 1, 2], P[:, 2, 2]], -1)
    w = np.exp(rng.uniform(np.log(1e-6), np.log(20.0), n)) * rng.choice([-1.0, 1.0], n)
    org = 8.0 * rng.integers(0, 32, (n, 3))
    reach = 4.0 + np.minimum(4.0 * s.max(1), 2000.0)
    m = org + 4.0 + rng.uniform(-1, 1, (n, 3)) * reach[:, None]
    if snap:
        m = np.floor(m) + rng.choice([0.0, 0.5], (n, 3))
    return np.concatenate([m, q, w[:, None], org], 1).astype(np.float32)


@pytest.fixture(scope="module")
def probe3(probe, tmp_path_factory):
    import glob
    lib = ctypes.CDLL(glob.glob(str(tmp_path_factory.getbasetemp() / "cull*" / "libcullprobe.so"))[0])
    lib.cull_probe3.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]

    def run(cases, boxes):
        cases = np.ascontiguousarray(cases, dtype=np.float32)
        boxes = np.ascontiguousarray(boxes, dtype=np.int32)
        out = np.zeros((len(cases), 4), dtype=np.int32)
        lib.cull_probe3(cases.ctypes.data, boxes.ctypes.data, len(cases), out.ctypes.data)
        return out

    return run


def _boxes3(rng, n, random_box):
    if not random_box:
        return np.tile(np.array([[0, 7, 0, 7, 0, 7]], np.int32), (n, 1))
    lo = rng.integers(0, 8, (n, 3))
    hi = np.minimum(lo + rng.integers(0, 8, (n, 3)), 7)
    return np.stack([lo[:, 0], hi[:, 0], lo[:, 1], hi[:, 1], lo[:, 2], hi[:, 2]], -1).astype(np.int32)


@pytest.mark.parametrize("kind", ["realistic", "tiny", "huge", "ill_conditioned", "snapped",
                                  "random_boxes"])
def test_brick_rows_never_drop_a_passing_voxel(probe3, kind):
    rng = np.random.default_rng(["realistic", "tiny", "huge", "ill_conditioned", "snapped",
                                 "random_boxes"].index(kind) + 31)
    n = 20000
    args = {"realistic": (0.3, 30.0), "tiny": (0.02, 0.5), "huge": (50.0, 2000.0),
            "ill_conditioned": (0.5, 50.0), "snapped": (0.3, 20.0),
            "random_boxes": (0.3, 30.0)}[kind]
    cases = _cases3(rng, n, *args, max_cond=1e6 if kind == "ill_conditioned" else None,
                    snap=kind == "snapped")
    out = probe3(cases, _boxes3(rng, n, kind == "random_boxes"))
    bad = np.nonzero(out[:, 0])[0]
    assert len(bad) == 0, f"{len(bad)} cases drop passing voxels, first: {cases[bad[0]]} -> {out[bad[0]]}"


def test_brick_rows_are_tight(probe3):
    rng = np.random.default_rng(7)
    n = 20000
    out = probe3(_cases3(rng, n, 1.0, 10.0), _boxes3(rng, n, False))
    live = out[:, 3] > 0
    assert (out[live, 2] >= out[live, 1]).all()
    # at most about one spare row per slice on average
    assert out[live, 2].mean() <= out[live, 1].mean() * 1.15 + 1.0
