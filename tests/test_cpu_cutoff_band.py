"""The rounding part of the cut-off bands (bt-3dgs_b200/csrc/r2s_cutoff.cuh),
checked on the CPU.

The backward kernels re-decide a pixel (voxel) with the reference's own test
when their shifted exponent z = s_thr - s lies within a band of the cut-off.
The band bounds |z - z_ref| by counting roundings: the kernels' float32 chain
for z is at most u (3 M + s_thr) from the exact value in 2D and u (4 M + 2 s_thr)
in 3D, plus its last rounding u |z| (negligible at the cut-off, where z ~ 0);
the reference's float32 sigma (in log2 units) at most 4 u M in 2D and 7 u M in
3D (u = 2^-24, M the magnitude of the quadratic's terms); the rest of the band
covers __expf and the threshold, whose error bounds are documented.
Here both float32 chains are evaluated operation for operation (products
rounded to float32, fused multiply-adds from exact float64 products) on random
conics up to a condition number of 1e4 and on points next to the cut-off, and
the measured errors are compared with those counts.  A fused multiply-add is
emulated by rounding the float64 sum of the exact product and the addend to
float32, which can differ from the true fma by one unit in the last place in
rare halfway cases; the measured maxima (0.78 of the 2D bound, 0.50 next to
the cut-off) leave room for it.
"""
import numpy as np

U = 2.0 ** -24
L = np.float64(np.float32(1.4426950408889634))  # kLog2e as the kernels store it


def f32(x):
    return np.asarray(x, dtype=np.float64).astype(np.float32)


def fma(a, b, c):
    return f32(np.float64(a) * np.float64(b) + np.float64(c))


def mul(a, b):
    return f32(np.float64(a) * np.float64(b))


def _conics_2d(rng, n):
    s1 = np.exp(rng.uniform(-1.0, 3.5, n))
    kappa = np.exp(rng.uniform(0.0, np.log(1e4), n))
    s2 = s1 / np.sqrt(kappa)
    th = rng.uniform(0, np.pi, n)
    c, s = np.cos(th), np.sin(th)
    cov = np.empty((n, 2, 2))
    cov[:, 0, 0] = c * c * s1 ** 2 + s * s * s2 ** 2
    cov[:, 1, 1] = s * s * s1 ** 2 + c * c * s2 ** 2
    cov[:, 0, 1] = cov[:, 1, 0] = c * s * (s1 ** 2 - s2 ** 2)
    P = np.linalg.inv(cov)
    return f32(P[:, 0, 0]), f32(P[:, 0, 1]), f32(P[:, 1, 1])


def test_2d_chains_stay_within_the_counted_roundings():
    rng = np.random.default_rng(0)
    n = 400_000
    a, b, c = _conics_2d(rng, n)
    wmu = np.exp(rng.uniform(np.log(2e-5), 0.0, n))
    s_thr = f32(np.log2(wmu * 1e5))
    # points at the cut-off (sigma = s_thr ln 2), jittered, and inside the ellipse
    A64, B64, C64 = np.float64(a), np.float64(b), np.float64(c)
    phi = rng.uniform(0, 2 * np.pi, n)
    dirx, diry = np.cos(phi), np.sin(phi)
    q = 0.5 * (A64 * dirx ** 2 + C64 * diry ** 2) + B64 * dirx * diry  # sigma per unit length^2
    r = np.sqrt(np.float64(s_thr) * np.log(2.0) / q) * rng.uniform(0.3, 1.02, n)
    dx, dy = f32(r * dirx), f32(r * diry)
    dx64, dy64 = np.float64(dx), np.float64(dy)
    # the kernels' chain (raster_bwd16_kernel): z = fma(dx, fma(A, dx, B dy), fma(Cc dy, dy, s_thr))
    A = mul(np.float32(-0.5 * L), a)
    B = mul(np.float32(-L), b)
    Cc = mul(np.float32(-0.5 * L), c)
    z = fma(dx, fma(A, dx, mul(B, dy)), fma(mul(Cc, dy), dy, s_thr))
    sig_exact = 0.5 * (A64 * dx64 ** 2 + C64 * dy64 ** 2) + B64 * dx64 * dy64
    z_exact = np.float64(s_thr) - L * sig_exact
    M = L * (0.5 * np.abs(A64) * dx64 ** 2 + np.abs(B64 * dx64 * dy64) + 0.5 * np.abs(C64) * dy64 ** 2)
    err_fast = np.abs(np.float64(z) - z_exact)
    bound_fast = U * (3 * M + np.abs(np.float64(s_thr)) + np.abs(np.float64(z)))
    assert np.all(err_fast <= bound_fast), float(np.max(err_fast / bound_fast))
    # the reference's sigma (ref_sigma2d_v2): fma(b dx, dy, 0.5 fma(a dx, dx, (c dy) dy))
    sig = fma(mul(b, dx), dy, mul(np.float32(0.5), fma(mul(a, dx), dx, mul(mul(c, dy), dy))))
    err_ref = np.abs(L * np.float64(sig) - L * sig_exact)
    assert np.all(err_ref <= U * 4 * M + L * U * np.abs(np.float64(sig))), (
        float(np.max(err_ref / (U * 4 * M))))
    # the points cover the cut-off region and ill-conditioned conics
    assert np.mean(np.abs(z_exact) < 0.05 * np.float64(s_thr)) > 0.05


def _conics_3d(rng, n):
    s = np.exp(rng.uniform(-1.0, 2.5, (n, 3)))
    s[:, 2] = s[:, 0] / np.sqrt(np.exp(rng.uniform(0.0, np.log(1e4), n)))
    q = rng.normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    R = np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                  2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                  2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
                 -1).reshape(n, 3, 3)
    cov = R @ (s[:, :, None] ** 2 * np.eye(3)) @ np.transpose(R, (0, 2, 1))
    P = np.linalg.inv(cov)
    return [f32(P[:, i, j]) for i, j in ((0, 0), (0, 1), (0, 2), (1, 1), (1, 2), (2, 2))]


def test_3d_chains_stay_within_the_counted_roundings():
    rng = np.random.default_rng(1)
    n = 300_000
    P00, P01, P02, P11, P12, P22 = _conics_3d(rng, n)
    w = np.exp(rng.uniform(np.log(2e-6), 0.0, n))
    s_thr = f32(np.log2(w * 1e6))
    d = rng.normal(size=(n, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    p64 = [np.float64(t) for t in (P00, P01, P02, P11, P12, P22)]
    qd = (0.5 * (p64[0] * d[:, 0] ** 2 + p64[3] * d[:, 1] ** 2 + p64[5] * d[:, 2] ** 2)
          + p64[1] * d[:, 0] * d[:, 1] + p64[2] * d[:, 0] * d[:, 2] + p64[4] * d[:, 1] * d[:, 2])
    r = np.sqrt(np.float64(s_thr) * np.log(2.0) / qd) * rng.uniform(0.3, 1.02, n)
    d1, d2, d3 = (f32(r * d[:, k]) for k in range(3))
    e1, e2, e3 = np.float64(d1), np.float64(d2), np.float64(d3)
    # the kernels' chain (voxel_bwd8_kernel): z = fma(dx, fma(A, dx, fma(B, dy, Cq dz)),
    #   fma(dy, fma(D, dy, E dz), fma(F dz, dz, s_thr)))
    h, o = np.float32(-0.5 * L), np.float32(-L)
    A, B, Cq = mul(h, P00), mul(o, P01), mul(o, P02)
    D, E, F = mul(h, P11), mul(o, P12), mul(h, P22)
    by = fma(B, d2, mul(Cq, d3))
    rest = fma(d2, fma(D, d2, mul(E, d3)), fma(mul(F, d3), d3, s_thr))
    z = fma(d1, fma(A, d1, by), rest)
    sig_exact = (0.5 * (p64[0] * e1 ** 2 + p64[3] * e2 ** 2 + p64[5] * e3 ** 2)
                 + p64[1] * e1 * e2 + p64[2] * e1 * e3 + p64[4] * e2 * e3)
    z_exact = np.float64(s_thr) - L * sig_exact
    M = L * (0.5 * np.abs(p64[0]) * e1 ** 2 + np.abs(p64[1] * e1 * e2) + np.abs(p64[2] * e1 * e3)
             + 0.5 * np.abs(p64[3]) * e2 ** 2 + np.abs(p64[4] * e2 * e3)
             + 0.5 * np.abs(p64[5]) * e3 ** 2)
    err_fast = np.abs(np.float64(z) - z_exact)
    bound_fast = U * (4 * M + 2 * np.abs(np.float64(s_thr)) + np.abs(np.float64(z)))
    assert np.all(err_fast <= bound_fast), float(np.max(err_fast / bound_fast))
    # the reference's sigma (ref_sigma3d variant 1)
    X = fma(mul(P22, d3), d3, fma(mul(P00, d1), d1, mul(mul(P11, d2), d2)))
    s1 = fma(mul(P01, d1), d2, mul(np.float32(0.5), X))
    s2 = fma(mul(P02, d1), d3, s1)
    sig = fma(mul(P12, d2), d3, s2)
    err_ref = np.abs(L * np.float64(sig) - L * sig_exact)
    assert np.all(err_ref <= U * 7 * M + L * U * np.abs(np.float64(sig))), (
        float(np.max(err_ref / (U * 7 * M))))
    assert np.mean(np.abs(z_exact) < 0.05 * np.float64(s_thr)) > 0.05
