// The reference's per-pixel and per-voxel cut-off expressions, restated.
//
// The reference keeps a (Gaussian, pixel) pair when sigma >= 0 and
// |alpha| >= 1e-5, with (csrc/RasterizeToPixelsFwd.cu:162-174,
// csrc/RasterizeToPixelsBwd.cu:423-430)
//   sigma = 0.5 * (a dx dx + c dy dy) + b dx dy,   alpha = (opacity mu) exp(-sigma)
// and a (Gaussian, voxel) pair when sigma >= 0 and |alpha| >= 1e-6, with
// (csrc/VoxelizeToVoxelsFwd.cu:196-210, csrc/VoxelizeToVoxelsBwd.cu:395-402)
//   sigma = 0.5 * (c00 d1 d1 + c11 d2 d2 + c22 d3 d3) + c01 d1 d2 + c02 d1 d3 + c12 d2 d3,
//   alpha = opacity exp(-sigma).
// Compiled with the same flags as the reference (fast math: exp of a float is
// the approximate exponential, and the compiler contracts products into
// fused multiply-adds), the same expression can still round differently if
// the compiler contracts it differently; the variants below fix the order of
// every rounding with explicit intrinsics, so that a test can find the one
// that reproduces the reference's values bit for bit
// (tests/test_gpu_refexpr.py).  The raster backward decides the pixels
// within rounding of the cut-off with ref_keep2d (r2s_raster.cu), the voxel
// backward the voxels with ref_keep3d (r2s_voxel.cu).
#pragma once

#include <cuda_runtime.h>

namespace r2s {

// 2D: sigma in the source's expression order, contracted by the compiler.
__device__ __forceinline__ float ref_sigma2d_src(float a, float b, float c, float dx, float dy) {
    return 0.5f * (a * dx * dx + c * dy * dy) + b * dx * dy;
}

// 2D: explicit rounding orders.  variant 1: fma(0.5, fma(a dx, dx, (c dy) dy), (b dx) dy)
__device__ __forceinline__ float ref_sigma2d_v1(float a, float b, float c, float dx, float dy) {
    const float cdy2 = __fmul_rn(__fmul_rn(c, dy), dy);
    const float x = __fmaf_rn(__fmul_rn(a, dx), dx, cdy2);
    return __fmaf_rn(0.5f, x, __fmul_rn(__fmul_rn(b, dx), dy));
}
// variant 2: fma(b dx, dy, 0.5 fma(a dx, dx, (c dy) dy))
__device__ __forceinline__ float ref_sigma2d_v2(float a, float b, float c, float dx, float dy) {
    const float cdy2 = __fmul_rn(__fmul_rn(c, dy), dy);
    const float x = __fmaf_rn(__fmul_rn(a, dx), dx, cdy2);
    return __fmaf_rn(__fmul_rn(b, dx), dy, __fmul_rn(0.5f, x));
}
// variant 3: fma(0.5, fma(c dy, dy, (a dx) dx), (b dx) dy)
__device__ __forceinline__ float ref_sigma2d_v3(float a, float b, float c, float dx, float dy) {
    const float adx2 = __fmul_rn(__fmul_rn(a, dx), dx);
    const float x = __fmaf_rn(__fmul_rn(c, dy), dy, adx2);
    return __fmaf_rn(0.5f, x, __fmul_rn(__fmul_rn(b, dx), dy));
}
// variant 4: fma(b dx, dy, 0.5 fma(c dy, dy, (a dx) dx))
__device__ __forceinline__ float ref_sigma2d_v4(float a, float b, float c, float dx, float dy) {
    const float adx2 = __fmul_rn(__fmul_rn(a, dx), dx);
    const float x = __fmaf_rn(__fmul_rn(c, dy), dy, adx2);
    return __fmaf_rn(__fmul_rn(b, dx), dy, __fmul_rn(0.5f, x));
}
// variant 5: no fusion at all
__device__ __forceinline__ float ref_sigma2d_v5(float a, float b, float c, float dx, float dy) {
    const float x = __fadd_rn(__fmul_rn(__fmul_rn(a, dx), dx), __fmul_rn(__fmul_rn(c, dy), dy));
    return __fadd_rn(__fmul_rn(0.5f, x), __fmul_rn(__fmul_rn(b, dx), dy));
}

__device__ __forceinline__ float ref_sigma2d(int variant, float a, float b, float c, float dx,
                                             float dy) {
    switch (variant) {
        case 1: return ref_sigma2d_v1(a, b, c, dx, dy);
        case 2: return ref_sigma2d_v2(a, b, c, dx, dy);
        case 3: return ref_sigma2d_v3(a, b, c, dx, dy);
        case 4: return ref_sigma2d_v4(a, b, c, dx, dy);
        case 5: return ref_sigma2d_v5(a, b, c, dx, dy);
        default: return ref_sigma2d_src(a, b, c, dx, dy);
    }
}

// alpha of a kept pair, 0 for a pair the reference drops
__device__ __forceinline__ float ref_alpha2d(int variant, float a, float b, float c, float wmu,
                                             float dx, float dy) {
    const float sigma = ref_sigma2d(variant, a, b, c, dx, dy);
    const float alpha = wmu * __expf(-sigma);
    return (sigma < 0.f || fabsf(alpha) < 1e-5f) ? 0.f : alpha;
}

// The reference's keep/drop decision for a (Gaussian, pixel) pair, bit for
// bit: variant 2, the one tests/test_gpu_refexpr.py finds exact for both the
// reference's forward and its backward.  wmu = opacity * mu (one rounded
// product, as the reference's `opac * mu * vis` forms it); dx, dy the pixel
// centre minus the mean.  A NaN alpha is kept, like the reference's test.
__device__ __forceinline__ bool ref_keep2d(float a, float b, float c, float wmu, float dx,
                                           float dy) {
    const float sigma = ref_sigma2d_v2(a, b, c, dx, dy);
    const float alpha = wmu * __expf(-sigma);
    return !(sigma < 0.f || fabsf(alpha) < 1e-5f);
}

// 3D: sigma = 0.5 (a d1 d1 + b d2 d2 + c d3 d3) + p d1 d2 + q d1 d3 + r d2 d3,
// alpha = opacity exp(-sigma), kept when sigma >= 0 and |alpha| >= 1e-6.
// Source order, contracted by the compiler.
__device__ __forceinline__ float ref_sigma3d_src(float a, float b, float c, float p, float q,
                                                 float r, float d1, float d2, float d3) {
    return 0.5f * (a * d1 * d1 + b * d2 * d2 + c * d3 * d3) + p * d1 * d2 + q * d1 * d3 +
           r * d2 * d3;
}

// the diagonal sum X with the first (variant bit 0 clear) or the second
// (bit 0 set) square contracted first, then the third square
__device__ __forceinline__ float ref_diag3d(int variant, float a, float b, float c, float d1,
                                           float d2, float d3) {
    const float x1 = (variant & 1)
                         ? __fmaf_rn(__fmul_rn(b, d2), d2, __fmul_rn(__fmul_rn(a, d1), d1))
                         : __fmaf_rn(__fmul_rn(a, d1), d1, __fmul_rn(__fmul_rn(b, d2), d2));
    return __fmaf_rn(__fmul_rn(c, d3), d3, x1);
}

// variants 1-4: bit 0 the diagonal order above; bit 1 clear: the half
// multiplied alone and the cross products contracted into it,
// fma(r d2, d3, fma(q d1, d3, fma(p d1, d2, 0.5 X))); bit 1 set: the half
// contracted with the first cross product, fma(0.5, X, (p d1) d2), then the
// other two.  variant 5: no fusion at all.
__device__ __forceinline__ float ref_sigma3d(int variant, float a, float b, float c, float p,
                                             float q, float r, float d1, float d2, float d3) {
    if (variant == 0) return ref_sigma3d_src(a, b, c, p, q, r, d1, d2, d3);
    if (variant == 5) {
        const float x = __fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(a, d1), d1),
                                            __fmul_rn(__fmul_rn(b, d2), d2)),
                                  __fmul_rn(__fmul_rn(c, d3), d3));
        float s = __fadd_rn(__fmul_rn(0.5f, x), __fmul_rn(__fmul_rn(p, d1), d2));
        s = __fadd_rn(s, __fmul_rn(__fmul_rn(q, d1), d3));
        return __fadd_rn(s, __fmul_rn(__fmul_rn(r, d2), d3));
    }
    const int v = variant - 1;
    const float x = ref_diag3d(v, a, b, c, d1, d2, d3);
    const float s1 = (v & 2) ? __fmaf_rn(0.5f, x, __fmul_rn(__fmul_rn(p, d1), d2))
                             : __fmaf_rn(__fmul_rn(p, d1), d2, __fmul_rn(0.5f, x));
    const float s2 = __fmaf_rn(__fmul_rn(q, d1), d3, s1);
    return __fmaf_rn(__fmul_rn(r, d2), d3, s2);
}

// The reference's keep/drop decision for a (Gaussian, voxel) pair, bit for
// bit: variant 1, the one tests/test_gpu_refexpr.py finds exact for the
// reference's voxelizer.  k = (c00, c01, c02, c11, c12, c22); d1, d2, d3 the
// voxel centre minus the mean.  A NaN alpha is kept, like the reference's test.
__device__ __forceinline__ bool ref_keep3d(const float k[6], float opac, float d1, float d2,
                                           float d3) {
    const float sigma = ref_sigma3d(1, k[0], k[3], k[5], k[1], k[2], k[4], d1, d2, d3);
    const float alpha = opac * __expf(-sigma);
    return !(sigma < 0.f || fabsf(alpha) < 1e-6f);
}

// alpha of a kept (Gaussian, voxel) pair, 0 for a pair the reference drops
__device__ __forceinline__ float ref_alpha3d(int variant, const float k[6], float opac, float d1,
                                             float d2, float d3) {
    // k = (c00, c01, c02, c11, c12, c22)
    const float sigma = ref_sigma3d(variant, k[0], k[3], k[5], k[1], k[2], k[4], d1, d2, d3);
    const float alpha = opac * __expf(-sigma);
    return (sigma < 0.f || fabsf(alpha) < 1e-6f) ? 0.f : alpha;
}

}  // namespace r2s
