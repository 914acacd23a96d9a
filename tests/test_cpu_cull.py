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
