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
// within rounding of the cut-off with ref_keep2d (r2s_raster.cu).
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

}  // namespace r2s
