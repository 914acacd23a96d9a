// Cut-off thresholds of the fast kernels and the bands around them inside
// which their decisions are re-checked against the reference's own test.
//
// The reference keeps a (Gaussian, pixel) pair when sigma >= 0 and
// |w mu exp(-sigma)| >= 1e-5, a (Gaussian, voxel) pair when sigma >= 0 and
// |w exp(-sigma)| >= 1e-6.  With s = sigma log2(e) that is 0 <= s <= s_thr,
// s_thr = log2(|w mu| 1e5) (2D) or log2(|w| 1e6) (3D).  The backward kernels
// evaluate the shifted exponent z = s_thr - s with pre-scaled coefficients
// and keep a pair when z >= 0; a pair with |z| <= delta (the band below) may
// be decided differently by the reference and is re-decided with
// ref_keep2d / ref_keep3d (r2s_refexpr.cuh); every other pair is decided
// alike by both tests.
#pragma once

#include <cuda_runtime.h>
#include <math_constants.h>

namespace r2s {

__device__ __forceinline__ float s_threshold(float wmu) {
    const float a = fabsf(wmu) * 1e5f;
    return a >= 1.0f ? log2f(a) : -1.0f;  // negative: nothing passes
}

__device__ __forceinline__ float s_threshold_v(float w) {
    const float a = fabsf(w) * 1e6f;
    return a >= 1.0f ? log2f(a) : -1.0f;  // records with a < 1 have an empty box
}

// 2D band.  Bound on |z - z_ref|, in log2 units with u = 2^-24 and
// M = log2(e) (|a| dx^2 / 2 + |b dx dy| + |c| dy^2 / 2) the magnitude of the
// quadratic's terms.  Each rounding of a partial result is at most u times
// that result; counted per term of the quadratic through the chains:
//   z = fma(dx, fma(A, dx, B dy), fma(Cc dy, dy, s_thr)), with the rounded
//     coefficients A, B, Cc: every term meets at most three roundings, s_thr
//     one (the last rounding, of a value near 0 at the cut-off, is negligible)
//                                                                 <= 3 u M + u s
//   reference sigma (ref_sigma2d_v2): every term meets at most four
//     roundings                                                       <= 4 u M
//   reference __expf(x), x ~ -s ln2: at most 2 + floor(1.173 |x|) ulp (the
//     CUDA intrinsic's documented bound), then alpha = w mu * vis (one ulp)
//                                                                 <= (7.3 + 2.4 s) u
//   threshold: |w mu| * 1e5 rounded, log2f (two units in the last place of
//     s_thr or 2^-21, whichever is larger), 1e-5f against 1/1e5    <= (4 s + 11) u
// i.e. |z - z_ref| <= u (7 M + 7.4 s_thr + 19); the band is about twice
// that, delta = u (16 M + 16 s_thr + 40).  M is bounded over the pixels that
// can lie near the cut-off: |dx| <= Dx, |dy| <= Dy, the record's culling
// extents (the ellipse at the cut-off, widened by margins for rounding) or
// any smaller bound on the offsets; a pixel outside the extents is dropped by
// both tests.
__device__ __forceinline__ float cutoff_band(float a, float b, float c, float s_thr, float Dx,
                                             float Dy) {
    const float M = 1.4426950408889634f * (0.5f * fabsf(a) * Dx * Dx + fabsf(b) * Dx * Dy +
                                           0.5f * fabsf(c) * Dy * Dy);
    const float d = (16.0f * M + 16.0f * fabsf(s_thr) + 40.0f) * 0x1p-24f;
    return d < 1e30f ? d : CUDART_INF_F;  // NaN: every pixel in the band
}

// 3D band, P = (P00, P01, P02, P11, P12, P22) the conic and M = log2(e)
// (|P00| dx^2 / 2 + |P01 dx dy| + |P02 dx dz| + |P11| dy^2 / 2 + |P12 dy dz|
// + |P22| dz^2 / 2).  Each rounding of a partial result is at most u times
// that result; counted per term of the quadratic through the chains:
//   z = fma(dx, fma(A, dx, fma(B, dy, Cq dz)), fma(dy, fma(D, dy, E dz),
//     fma(F dz, dz, s_thr))), with the rounded coefficients A .. F: every
//     term meets at most four roundings, s_thr two                <= 4 u M + 2 u s
//   reference sigma (variant 1 of ref_sigma3d): every term meets at most
//     seven roundings                                                 <= 7 u M
//   reference __expf(x), x ~ -s ln2 (at most 2 + floor(1.173 |x|) ulp, the
//     intrinsic's documented bound), alpha = w * vis              <= (7.3 + 2.4 s) u
//   threshold: |w| * 1e6 rounded, log2f (two units in the last place of s_thr
//     or 2^-21, whichever is larger), 1e-6f against 1/1e6         <= (4 s + 11) u
// i.e. |z - z_ref| <= u (11 M + 8.4 s_thr + 19); the band is about twice
// that, delta = u (24 M + 18 s_thr + 48), with |dx|, |dy|, |dz| bounded by
// the culling extents (Dx, Dy, Dz).
__device__ __forceinline__ float cutoff_band_v(const float P[6], float s_thr, float Dx, float Dy,
                                               float Dz) {
    const float M = 1.4426950408889634f *
                    (0.5f * fabsf(P[0]) * Dx * Dx + fabsf(P[1]) * Dx * Dy + fabsf(P[2]) * Dx * Dz +
                     0.5f * fabsf(P[3]) * Dy * Dy + fabsf(P[4]) * Dy * Dz + 0.5f * fabsf(P[5]) * Dz * Dz);
    const float d = (24.0f * M + 18.0f * fabsf(s_thr) + 48.0f) * 0x1p-24f;
    return d < 1e30f ? d : CUDART_INF_F;  // NaN, infinite extents: every voxel in the band
}

}  // namespace r2s
