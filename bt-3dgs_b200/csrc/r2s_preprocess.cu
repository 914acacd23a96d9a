// Per-Gaussian and per-(view, Gaussian) preprocessing: parameter transform,
// cone-beam projection, conics/mu, world->volume mapping, their VJPs, the
// fused splat-record producers and the fused per-Gaussian explicit backward.
//
// Bit-exactness note.  Radii and tile rectangles are integer outputs that
// must equal the reference's.  They are derived from floating-point chains
// (covariance from quaternion/scale, projected covariance, mapped
// covariance), so those chains are written with the same expression trees as
// the reference kernels and compiled with the same flags (-O3
// --use_fast_math, FMA contraction on): the same association order gives the
// same FMA contraction and hence the same rounding.  The functions that must
// stay in this form are marked "expression order fixed".
#include <math_constants.h>

#include "r2s_common.cuh"
#include "r2s_cutoff.cuh"
#include "r2s_tiles.cuh"

namespace r2s {

// ===========================================================================
// Parameter transform  (reference: csrc/ParameterTransformFwd.cu:52-129,
// csrc/ParameterTransformBwd.cu:65-245)
// ===========================================================================

// Normalized quaternion -> rotation matrix rows and activated scales.
// Expression order fixed (ParameterTransformFwd.cu:66-107).
template <typename S>
struct RotScale {
    S w, x, y, z;        // normalized quaternion
    S qnorm, inv_qnorm;  // ||q_raw||, 1 / max(||q_raw||, 1e-12)
    S R[3][3];
    S s[3], sig[3];
};

template <typename S>
__device__ __forceinline__ void rot_scale(const S* __restrict__ q4, const S* __restrict__ so3,
                                          S scale_min, S scale_max, RotScale<S>& o) {
    const S qw = q4[0], qx = q4[1], qy = q4[2], qz = q4[3];
    o.qnorm = sqrt(qw * qw + qx * qx + qy * qy + qz * qz);
    o.inv_qnorm = static_cast<S>(1) / max(o.qnorm, static_cast<S>(1e-12));
    o.w = qw * o.inv_qnorm;
    o.x = qx * o.inv_qnorm;
    o.y = qy * o.inv_qnorm;
    o.z = qz * o.inv_qnorm;
    const S span = scale_max - scale_min;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const S raw = so3[i];
        o.sig[i] = static_cast<S>(1) / (static_cast<S>(1) + exp(-raw));
        o.s[i] = o.sig[i] * span + scale_min;
    }
    const S xx = o.x * o.x, yy = o.y * o.y, zz = o.z * o.z;
    const S xy = o.x * o.y, xz = o.x * o.z, yz = o.y * o.z;
    const S wx = o.w * o.x, wy = o.w * o.y, wz = o.w * o.z;
    o.R[0][0] = static_cast<S>(1) - static_cast<S>(2) * (yy + zz);
    o.R[0][1] = static_cast<S>(2) * (xy - wz);
    o.R[0][2] = static_cast<S>(2) * (xz + wy);
    o.R[1][0] = static_cast<S>(2) * (xy + wz);
    o.R[1][1] = static_cast<S>(1) - static_cast<S>(2) * (xx + zz);
    o.R[1][2] = static_cast<S>(2) * (yz - wx);
    o.R[2][0] = static_cast<S>(2) * (xz - wy);
    o.R[2][1] = static_cast<S>(2) * (yz + wx);
    o.R[2][2] = static_cast<S>(1) - static_cast<S>(2) * (xx + yy);
}

// Sigma = R diag(s^2) R^T, upper triangle.  Expression order fixed
// (ParameterTransformFwd.cu:110-119).
template <typename S>
__device__ __forceinline__ void covar_from(const RotScale<S>& o, S cov[6]) {
    const S q0 = o.s[0] * o.s[0], q1 = o.s[1] * o.s[1], q2 = o.s[2] * o.s[2];
    const S(&R)[3][3] = o.R;
    cov[0] = R[0][0] * R[0][0] * q0 + R[0][1] * R[0][1] * q1 + R[0][2] * R[0][2] * q2;
    cov[1] = R[0][0] * R[1][0] * q0 + R[0][1] * R[1][1] * q1 + R[0][2] * R[1][2] * q2;
    cov[2] = R[0][0] * R[2][0] * q0 + R[0][1] * R[2][1] * q1 + R[0][2] * R[2][2] * q2;
    cov[3] = R[1][0] * R[1][0] * q0 + R[1][1] * R[1][1] * q1 + R[1][2] * R[1][2] * q2;
    cov[4] = R[1][0] * R[2][0] * q0 + R[1][1] * R[2][1] * q1 + R[1][2] * R[2][2] * q2;
    cov[5] = R[2][0] * R[2][0] * q0 + R[2][1] * R[2][1] * q1 + R[2][2] * R[2][2] * q2;
}

// VJP of covar_from through the normalization and the bounded sigmoid
// (ParameterTransformBwd.cu:116-244): off-diagonal cotangents are halved to
// form the symmetric cotangent, then dL/dR = 2 V R S^2, dL/ds_j =
// sum_i R_ij (2 V R S)_ij, and the quaternion VJP of the rotation matrix.
template <typename S>
__device__ __forceinline__ void covar_vjp(const RotScale<S>& o, const S vc[6], S scale_min,
                                          S scale_max, S v_q[4], S v_so[3]) {
    const S(&R)[3][3] = o.R;
    const S h = static_cast<S>(0.5);
    const S V[3][3] = {{vc[0], vc[1] * h, vc[2] * h},
                       {vc[1] * h, vc[3], vc[4] * h},
                       {vc[2] * h, vc[4] * h, vc[5]}};
    // VR[i][j] = sum_k V[i][k] R[k][j]
    S VR[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) VR[i][j] = V[i][0] * R[0][j] + V[i][1] * R[1][j] + V[i][2] * R[2][j];
    S vM[3][3], vR[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            vM[i][j] = static_cast<S>(2) * VR[i][j] * o.s[j];
            vR[i][j] = static_cast<S>(2) * VR[i][j] * o.s[j] * o.s[j];
        }
    const S w = o.w, x = o.x, y = o.y, z = o.z;
    const S gw = static_cast<S>(2) * (x * (vR[2][1] - vR[1][2]) + y * (vR[0][2] - vR[2][0]) +
                                      z * (vR[1][0] - vR[0][1]));
    const S gx = static_cast<S>(2) * (static_cast<S>(-2) * x * (vR[1][1] + vR[2][2]) +
                                      y * (vR[0][1] + vR[1][0]) + z * (vR[0][2] + vR[2][0]) +
                                      w * (vR[2][1] - vR[1][2]));
    const S gy = static_cast<S>(2) * (x * (vR[0][1] + vR[1][0]) +
                                      static_cast<S>(-2) * y * (vR[0][0] + vR[2][2]) +
                                      z * (vR[1][2] + vR[2][1]) + w * (vR[0][2] - vR[2][0]));
    const S gz = static_cast<S>(2) * (x * (vR[0][2] + vR[2][0]) + y * (vR[1][2] + vR[2][1]) +
                                      static_cast<S>(-2) * z * (vR[0][0] + vR[1][1]) +
                                      w * (vR[1][0] - vR[0][1]));
    const S span = scale_max - scale_min;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const S vs = R[0][j] * vM[0][j] + R[1][j] * vM[1][j] + R[2][j] * vM[2][j];
        v_so[j] = vs * o.sig[j] * (static_cast<S>(1) - o.sig[j]) * span;
    }
    if (o.qnorm > static_cast<S>(1e-12)) {
        const S dot = w * gw + x * gx + y * gy + z * gz;
        v_q[0] = (gw - w * dot) * o.inv_qnorm;
        v_q[1] = (gx - x * dot) * o.inv_qnorm;
        v_q[2] = (gy - y * dot) * o.inv_qnorm;
        v_q[3] = (gz - z * dot) * o.inv_qnorm;
    } else {
        v_q[0] = gw * o.inv_qnorm;
        v_q[1] = gx * o.inv_qnorm;
        v_q[2] = gy * o.inv_qnorm;
        v_q[3] = gz * o.inv_qnorm;
    }
}

template <typename S>
__global__ void param_fwd_kernel(const S* __restrict__ quats, const S* __restrict__ so,
                                 S smin, S smax, S* __restrict__ covars,
                                 S* __restrict__ max_scales, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    RotScale<S> o;
    rot_scale(quats + i * 4, so + i * 3, smin, smax, o);
    max_scales[i] = max(o.s[0], max(o.s[1], o.s[2]));
    S cov[6];
    covar_from(o, cov);
#pragma unroll
    for (int k = 0; k < 6; ++k) covars[i * 6 + k] = cov[k];
}

template <typename S>
__global__ void param_bwd_kernel(const S* __restrict__ quats, const S* __restrict__ so,
                                 S smin, S smax, const S* __restrict__ v_covars,
                                 S* __restrict__ v_quats, S* __restrict__ v_so, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    RotScale<S> o;
    rot_scale(quats + i * 4, so + i * 3, smin, smax, o);
    S vc[6], vq[4], vs[3];
#pragma unroll
    for (int k = 0; k < 6; ++k) vc[k] = v_covars[i * 6 + k];
    covar_vjp(o, vc, smin, smax, vq, vs);
#pragma unroll
    for (int k = 0; k < 4; ++k) v_quats[i * 4 + k] = vq[k];
#pragma unroll
    for (int k = 0; k < 3; ++k) v_so[i * 3 + k] = vs[k];
}

// softplus / sigmoid evaluated in double so that the float result matches
// torch.nn.functional.softplus(beta=1, threshold=20) and torch.sigmoid to
// rounding (the library is built with fast-math, whose expf is approximate).
__device__ __forceinline__ float softplus_f(float x) {
    if (x > 20.0f) return x;
    return static_cast<float>(log1p(exp(static_cast<double>(x))));
}
__device__ __forceinline__ float sigmoid_f(float x) {
    return static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(x))));
}

// Parameter transform of the fused path (covariances and max scales); the
// opacities come from launch_softplus_f32 (r2s_precise.cu), which matches
// torch.nn.functional.softplus bit for bit.
__global__ void prepare_kernel(const float* __restrict__ quats, const float* __restrict__ so,
                               float smin, float smax, float* __restrict__ covars,
                               float* __restrict__ max_scales, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    RotScale<float> o;
    rot_scale(quats + i * 4, so + i * 3, smin, smax, o);
    max_scales[i] = fmaxf(o.s[0], fmaxf(o.s[1], o.s[2]));
    float cov[6];
    covar_from(o, cov);
#pragma unroll
    for (int k = 0; k < 6; ++k) covars[i * 6 + k] = cov[k];
}

// ===========================================================================
// Cone-beam projection  (reference: csrc/WorldToImageProjectionFwd.cu:73-283)
// ===========================================================================

template <typename S>
struct View {
    S R00, R01, R02, R10, R11, R12, R20, R21, R22;
    S t0, t1, t2;
    S fx, fy, cx, cy;
};

template <typename S>
__device__ __forceinline__ View<S> load_view(const S* __restrict__ viewmats,
                                             const S* __restrict__ Ks, int64_t c) {
    const S* m = viewmats + c * 16;
    const S* k = Ks + c * 9;
    View<S> v;
    v.R00 = m[0]; v.R01 = m[1]; v.R02 = m[2]; v.t0 = m[3];
    v.R10 = m[4]; v.R11 = m[5]; v.R12 = m[6]; v.t1 = m[7];
    v.R20 = m[8]; v.R21 = m[9]; v.R22 = m[10]; v.t2 = m[11];
    v.fx = k[0]; v.fy = k[4]; v.cx = k[2]; v.cy = k[5];
    return v;
}

// Everything the forward and backward need about one (view, Gaussian) pair.
// Expression order fixed (WorldToImageProjectionFwd.cu:124-231 and the
// identical recomputation in WorldToImageProjectionBwd.cu:112-196).
template <typename S>
struct ProjState {
    S x, y, z;
    S rz, rz2;
    S xrz, yrz, tx, ty;
    bool x_clipped, y_clipped;
    S l, rl;
    S J00, J02, J11, J12, J20, J21, J22;
    S Sc00, Sc01, Sc02, Sc11, Sc12, Sc22;
    S mx, my;
    S C[6];  // projected 3x3 covariance, upper triangle
};

template <typename S>
__device__ __forceinline__ bool project_state(const View<S>& v, S px, S py, S pz,
                                              const S* __restrict__ cov3, S W, S H,
                                              ProjState<S>& p) {
    p.x = v.R00 * px + v.R01 * py + v.R02 * pz + v.t0;
    p.y = v.R10 * px + v.R11 * py + v.R12 * pz + v.t1;
    p.z = v.R20 * px + v.R21 * py + v.R22 * pz + v.t2;
    if (p.z <= static_cast<S>(0.01)) return false;
    p.rz = static_cast<S>(1) / p.z;
    p.rz2 = p.rz * p.rz;
    p.mx = v.fx * p.x * p.rz + v.cx;
    p.my = v.fy * p.y * p.rz + v.cy;

    const S tan_fovx = static_cast<S>(0.5) * W / v.fx;
    const S tan_fovy = static_cast<S>(0.5) * H / v.fy;
    const S lim_x_pos = (W - v.cx) / v.fx + static_cast<S>(0.3) * tan_fovx;
    const S lim_x_neg = v.cx / v.fx + static_cast<S>(0.3) * tan_fovx;
    const S lim_y_pos = (H - v.cy) / v.fy + static_cast<S>(0.3) * tan_fovy;
    const S lim_y_neg = v.cy / v.fy + static_cast<S>(0.3) * tan_fovy;
    p.xrz = p.x * p.rz;
    p.yrz = p.y * p.rz;
    p.tx = p.z * min(lim_x_pos, max(-lim_x_neg, p.xrz));
    p.ty = p.z * min(lim_y_pos, max(-lim_y_neg, p.yrz));
    p.x_clipped = (p.xrz > lim_x_pos) || (p.xrz < -lim_x_neg);
    p.y_clipped = (p.yrz > lim_y_pos) || (p.yrz < -lim_y_neg);

    p.l = sqrt(p.tx * p.tx + p.ty * p.ty + p.z * p.z);
    p.rl = static_cast<S>(1) / p.l;
    p.J00 = v.fx * p.rz;
    p.J02 = -v.fx * p.tx * p.rz2;
    p.J11 = v.fy * p.rz;
    p.J12 = -v.fy * p.ty * p.rz2;
    p.J20 = p.tx * p.rl;
    p.J21 = p.ty * p.rl;
    p.J22 = p.z * p.rl;

    const S s00 = cov3[0], s01 = cov3[1], s02 = cov3[2];
    const S s11 = cov3[3], s12 = cov3[4], s22 = cov3[5];
    // M = Sigma R^T
    const S M00 = s00 * v.R00 + s01 * v.R01 + s02 * v.R02;
    const S M01 = s00 * v.R10 + s01 * v.R11 + s02 * v.R12;
    const S M02 = s00 * v.R20 + s01 * v.R21 + s02 * v.R22;
    const S M10 = s01 * v.R00 + s11 * v.R01 + s12 * v.R02;
    const S M11 = s01 * v.R10 + s11 * v.R11 + s12 * v.R12;
    const S M12 = s01 * v.R20 + s11 * v.R21 + s12 * v.R22;
    const S M20 = s02 * v.R00 + s12 * v.R01 + s22 * v.R02;
    const S M21 = s02 * v.R10 + s12 * v.R11 + s22 * v.R12;
    const S M22 = s02 * v.R20 + s12 * v.R21 + s22 * v.R22;
    // Sigma_c = R M
    p.Sc00 = v.R00 * M00 + v.R01 * M10 + v.R02 * M20;
    p.Sc01 = v.R00 * M01 + v.R01 * M11 + v.R02 * M21;
    p.Sc02 = v.R00 * M02 + v.R01 * M12 + v.R02 * M22;
    p.Sc11 = v.R10 * M01 + v.R11 * M11 + v.R12 * M21;
    p.Sc12 = v.R10 * M02 + v.R11 * M12 + v.R12 * M22;
    p.Sc22 = v.R20 * M02 + v.R21 * M12 + v.R22 * M22;
    // Nm = Sigma_c J^T (the zero entries of J kept as written in the reference
    // so that the contraction pattern, hence the rounding, is the same)
    const S zero = static_cast<S>(0);
    const S N00 = p.Sc00 * p.J00 + p.Sc02 * p.J02;
    const S N01 = p.Sc00 * zero + p.Sc01 * p.J11 + p.Sc02 * p.J12;
    const S N02 = p.Sc00 * p.J20 + p.Sc01 * p.J21 + p.Sc02 * p.J22;
    const S N10 = p.Sc01 * p.J00 + p.Sc12 * p.J02;
    const S N11 = p.Sc01 * zero + p.Sc11 * p.J11 + p.Sc12 * p.J12;
    const S N12 = p.Sc01 * p.J20 + p.Sc11 * p.J21 + p.Sc12 * p.J22;
    const S N20 = p.Sc02 * p.J00 + p.Sc22 * p.J02;
    const S N21 = p.Sc02 * zero + p.Sc12 * p.J11 + p.Sc22 * p.J12;
    const S N22 = p.Sc02 * p.J20 + p.Sc12 * p.J21 + p.Sc22 * p.J22;
    (void)N10;
    // C2 = J Nm
    p.C[0] = p.J00 * N00 + p.J02 * N20;
    p.C[1] = p.J00 * N01 + p.J02 * N21;
    p.C[2] = p.J00 * N02 + p.J02 * N22;
    p.C[3] = p.J11 * N11 + p.J12 * N21;
    p.C[4] = p.J11 * N12 + p.J12 * N22;
    p.C[5] = p.J20 * N02 + p.J21 * N12 + p.J22 * N22;
    return true;
}

// Rectangular radii with culling (WorldToImageProjectionFwd.cu:250-282).
// Expression order fixed.  Returns false (radii 0) when culled.
template <typename S>
__device__ __forceinline__ bool image_radii(const S C[6], S mx, S my, S eps, S clip,
                                            uint32_t width, uint32_t height, int32_t& rx,
                                            int32_t& ry) {
    const S a_blur = C[0] + eps;
    const S d_blur = C[3] + eps;
    const S b_off = C[1];
    const S det_blur = a_blur * d_blur - b_off * b_off;
    rx = 0;
    ry = 0;
    if (det_blur <= static_cast<S>(0)) return false;
    const S rad_x = ceil(clip * sqrt(max(static_cast<S>(0), a_blur)));
    const S rad_y = ceil(clip * sqrt(max(static_cast<S>(0), d_blur)));
    if (!isfinite(rad_x) || !isfinite(rad_y) || rad_x <= static_cast<S>(0) ||
        rad_y <= static_cast<S>(0))
        return false;
    if (mx + rad_x <= static_cast<S>(0) || mx - rad_x >= static_cast<S>(width) ||
        my + rad_y <= static_cast<S>(0) || my - rad_y >= static_cast<S>(height))
        return false;
    rx = static_cast<int32_t>(rad_x);
    ry = static_cast<int32_t>(rad_y);
    return true;
}

// Conic and mu of a projected covariance (ConicsMuFwd.cu:55-99).
template <typename S>
__device__ __forceinline__ bool conic_mu(const S C[6], S eps, S& u11, S& u12, S& u22, S& mu) {
    const S a = C[0], b = C[1], c = C[2], d = C[3], e = C[4], f = C[5];
    const S ab = a + eps;
    const S db = d + eps;
    const S fb = f + eps;
    const S D2b = ab * db - b * b;
    const S D3b = ab * db * fb - ab * e * e - b * b * fb + static_cast<S>(2) * b * c * e - c * c * db;
    if (D2b <= static_cast<S>(1e-9)) {
        u11 = u12 = u22 = mu = static_cast<S>(0);
        return false;
    }
    const S inv = static_cast<S>(1) / D2b;
    u11 = db * inv;
    u12 = -b * inv;
    u22 = ab * inv;
    const S ratio = D3b * inv;
    mu = ratio > static_cast<S>(0) ? sqrt(static_cast<S>(2.0 * CUDART_PI) * ratio)
                                   : static_cast<S>(0);
    return true;
}

// VJP of conic_mu (ConicsMuBwd.cu:70-161): conic part -P dV P on the
// independent entries and mu part (mu/2)(Q - pad(P)) with Q = inverse of the
// blurred 3x3 covariance.
template <typename S>
__device__ __forceinline__ void conic_mu_vjp(const S C[6], S eps, S u11, S u12, S u22, S mu,
                                             S vu11, S vu12, S vu22, S vmu, S g[6]) {
    if (u11 == static_cast<S>(0) && u12 == static_cast<S>(0) && u22 == static_cast<S>(0)) {
#pragma unroll
        for (int k = 0; k < 6; ++k) g[k] = static_cast<S>(0);
        return;
    }
    g[0] = -(vu11 * u11 * u11 + vu12 * u11 * u12 + vu22 * u12 * u12);
    g[1] = -(vu11 * static_cast<S>(2) * u11 * u12 + vu12 * (u11 * u22 + u12 * u12) +
             vu22 * static_cast<S>(2) * u12 * u22);
    g[2] = static_cast<S>(0);
    g[3] = -(vu11 * u12 * u12 + vu12 * u12 * u22 + vu22 * u22 * u22);
    g[4] = static_cast<S>(0);
    g[5] = static_cast<S>(0);
    if (mu > static_cast<S>(0)) {
        const S ab = C[0] + eps, b = C[1], c = C[2], db = C[3] + eps, e = C[4], fb = C[5] + eps;
        const S D3b =
            ab * db * fb - ab * e * e - b * b * fb + static_cast<S>(2) * b * c * e - c * c * db;
        if (D3b > static_cast<S>(1e-9)) {
            const S inv = static_cast<S>(1) / D3b;
            const S q00 = (db * fb - e * e) * inv;
            const S q01 = (c * e - b * fb) * inv;
            const S q02 = (b * e - c * db) * inv;
            const S q11 = (ab * fb - c * c) * inv;
            const S q12 = (b * c - ab * e) * inv;
            const S q22 = (ab * db - b * b) * inv;
            const S hv = static_cast<S>(0.5) * mu * vmu;
            g[0] += hv * (q00 - u11);
            g[1] += hv * (static_cast<S>(2) * q01 - static_cast<S>(2) * u12);
            g[2] += hv * (static_cast<S>(2) * q02);
            g[3] += hv * (q11 - u22);
            g[4] += hv * (static_cast<S>(2) * q12);
            g[5] += hv * q22;
        }
    }
}

// VJP of the projection for one (view, Gaussian): cotangents of means2d and
// of the 6 stored entries of the projected covariance -> world mean and the
// 6 stored covariance entries.  Follows WorldToImageProjectionBwd.cu:200-541
// including its treatment of the FOV-clamped branches.
template <typename S>
__device__ __forceinline__ void project_vjp(const View<S>& v, const ProjState<S>& p, S vmx,
                                            S vmy, const S G[6], S v_p[3], S v_s[6]) {
    const S rz3 = p.rz2 * p.rz;
    const S rl2 = p.rl * p.rl;
    const S va = G[0], vb = G[1], vcc = G[2], vd = G[3], ve = G[4], vf = G[5];
    const S J00 = p.J00, J02 = p.J02, J11 = p.J11, J12 = p.J12, J20 = p.J20, J21 = p.J21,
            J22 = p.J22;

    S vpx = v.fx * p.rz * vmx;
    S vpy = v.fy * p.rz * vmy;
    S vpz = -(v.fx * p.x * p.rz2 * vmx + v.fy * p.y * p.rz2 * vmy);

    // covariance path: vSc = J^T Gu J (Gu upper triangular), vS = R^T vSc R
    const S T00 = va * J00 + vcc * J20;
    const S T01 = vb * J11 + vcc * J21;
    const S T02 = va * J02 + vb * J12 + vcc * J22;
    const S T10 = ve * J20;
    const S T11 = vd * J11 + ve * J21;
    const S T12 = vd * J12 + ve * J22;
    const S T20 = vf * J20;
    const S T21 = vf * J21;
    const S T22 = vf * J22;
    const S A00 = J00 * T00 + J20 * T20, A01 = J00 * T01 + J20 * T21, A02 = J00 * T02 + J20 * T22;
    const S A10 = J11 * T10 + J21 * T20, A11 = J11 * T11 + J21 * T21, A12 = J11 * T12 + J21 * T22;
    const S A20 = J02 * T00 + J12 * T10 + J22 * T20;
    const S A21 = J02 * T01 + J12 * T11 + J22 * T21;
    const S A22 = J02 * T02 + J12 * T12 + J22 * T22;
    const S Q00 = A00 * v.R00 + A01 * v.R10 + A02 * v.R20;
    const S Q01 = A00 * v.R01 + A01 * v.R11 + A02 * v.R21;
    const S Q02 = A00 * v.R02 + A01 * v.R12 + A02 * v.R22;
    const S Q10 = A10 * v.R00 + A11 * v.R10 + A12 * v.R20;
    const S Q11 = A10 * v.R01 + A11 * v.R11 + A12 * v.R21;
    const S Q12 = A10 * v.R02 + A11 * v.R12 + A12 * v.R22;
    const S Q20 = A20 * v.R00 + A21 * v.R10 + A22 * v.R20;
    const S Q21 = A20 * v.R01 + A21 * v.R11 + A22 * v.R21;
    const S Q22 = A20 * v.R02 + A21 * v.R12 + A22 * v.R22;
    const S vS00 = v.R00 * Q00 + v.R10 * Q10 + v.R20 * Q20;
    const S vS01 = v.R00 * Q01 + v.R10 * Q11 + v.R20 * Q21;
    const S vS02 = v.R00 * Q02 + v.R10 * Q12 + v.R20 * Q22;
    const S vS10 = v.R01 * Q00 + v.R11 * Q10 + v.R21 * Q20;
    const S vS11 = v.R01 * Q01 + v.R11 * Q11 + v.R21 * Q21;
    const S vS12 = v.R01 * Q02 + v.R11 * Q12 + v.R21 * Q22;
    const S vS20 = v.R02 * Q00 + v.R12 * Q10 + v.R22 * Q20;
    const S vS21 = v.R02 * Q01 + v.R12 * Q11 + v.R22 * Q21;
    const S vS22 = v.R02 * Q02 + v.R12 * Q12 + v.R22 * Q22;
    v_s[0] = vS00;
    v_s[1] = vS01 + vS10;
    v_s[2] = vS02 + vS20;
    v_s[3] = vS11;
    v_s[4] = vS12 + vS21;
    v_s[5] = vS22;

    // Jacobian path: vJ = (Gu + Gu^T) J Sigma_c
    const S U00 = J00 * p.Sc00 + J02 * p.Sc02;
    const S U01 = J00 * p.Sc01 + J02 * p.Sc12;
    const S U02 = J00 * p.Sc02 + J02 * p.Sc22;
    const S U10 = J11 * p.Sc01 + J12 * p.Sc02;
    const S U11 = J11 * p.Sc11 + J12 * p.Sc12;
    const S U12 = J11 * p.Sc12 + J12 * p.Sc22;
    const S U20 = J20 * p.Sc00 + J21 * p.Sc01 + J22 * p.Sc02;
    const S U21 = J20 * p.Sc01 + J21 * p.Sc11 + J22 * p.Sc12;
    const S U22 = J20 * p.Sc02 + J21 * p.Sc12 + J22 * p.Sc22;
    const S two = static_cast<S>(2);
    const S vJ00 = two * va * U00 + vb * U10 + vcc * U20;
    const S vJ02 = two * va * U02 + vb * U12 + vcc * U22;
    const S vJ11 = vb * U01 + two * vd * U11 + ve * U21;
    const S vJ12 = vb * U02 + two * vd * U12 + ve * U22;
    const S vJ20 = vcc * U00 + ve * U10 + two * vf * U20;
    const S vJ21 = vcc * U01 + ve * U11 + two * vf * U21;
    const S vJ22 = vcc * U02 + ve * U12 + two * vf * U22;

    const S tx = p.tx, ty = p.ty, z = p.z, rl = p.rl;
    vpz += -v.fx * p.rz2 * vJ00;
    vpz += -v.fy * p.rz2 * vJ11;
    vpz += rl * vJ22;
    if (!p.x_clipped) vpx += -v.fx * p.rz2 * vJ02;
    vpz += two * v.fx * tx * rz3 * vJ02;
    if (!p.y_clipped) vpy += -v.fy * p.rz2 * vJ12;
    vpz += two * v.fy * ty * rz3 * vJ12;
    if (!p.x_clipped) vpx += rl * vJ20;
    if (!p.y_clipped) vpy += rl * vJ21;
    const S v_l = -tx * rl2 * vJ20 - ty * rl2 * vJ21 - z * rl2 * vJ22;
    if (!p.x_clipped) vpx += v_l * tx * rl;
    if (!p.y_clipped) vpy += v_l * ty * rl;
    vpz += v_l * z * rl;
    if (p.x_clipped) {
        vpz += v_l * tx * rl * (tx / z);
        vpz += (tx / z) * rl * vJ20;
    }
    if (p.y_clipped) {
        vpz += v_l * ty * rl * (ty / z);
        vpz += (ty / z) * rl * vJ21;
    }
    if (p.x_clipped) vpz += -v.fx * (tx / z) * p.rz2 * vJ02;
    if (p.y_clipped) vpz += -v.fy * (ty / z) * p.rz2 * vJ12;

    v_p[0] = v.R00 * vpx + v.R10 * vpy + v.R20 * vpz;
    v_p[1] = v.R01 * vpx + v.R11 * vpy + v.R21 * vpz;
    v_p[2] = v.R02 * vpx + v.R12 * vpy + v.R22 * vpz;
}

template <typename S>
__global__ void project_fwd_kernel(const S* __restrict__ means, const S* __restrict__ covars,
                                   const S* __restrict__ viewmats, const S* __restrict__ Ks,
                                   int64_t C, int64_t N, uint32_t width, uint32_t height, S eps,
                                   S clip, S* __restrict__ means2d, S* __restrict__ cov2d,
                                   int32_t* __restrict__ radii) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= C * N) return;
    const int64_t c = idx / N, g = idx - c * N;
    const View<S> v = load_view(viewmats, Ks, c);
    ProjState<S> p;
    const bool front = project_state(v, means[g * 3], means[g * 3 + 1], means[g * 3 + 2],
                                     covars + g * 6, static_cast<S>(width),
                                     static_cast<S>(height), p);
    if (!front) {
        means2d[idx * 2] = means2d[idx * 2 + 1] = static_cast<S>(0);
#pragma unroll
        for (int k = 0; k < 6; ++k) cov2d[idx * 6 + k] = static_cast<S>(0);
        radii[idx * 2] = radii[idx * 2 + 1] = 0;
        return;
    }
    means2d[idx * 2] = p.mx;
    means2d[idx * 2 + 1] = p.my;
#pragma unroll
    for (int k = 0; k < 6; ++k) cov2d[idx * 6 + k] = p.C[k];
    int32_t rx, ry;
    image_radii(p.C, p.mx, p.my, eps, clip, width, height, rx, ry);
    radii[idx * 2] = rx;
    radii[idx * 2 + 1] = ry;
}

// Thread per Gaussian, loop over views: the per-view contributions are summed
// in registers (the reference accumulates them with 9 float atomics per pair,
// WorldToImageProjectionBwd.cu:548-553).
template <typename S>
__global__ void project_bwd_kernel(const S* __restrict__ means, const S* __restrict__ covars,
                                   const S* __restrict__ viewmats, const S* __restrict__ Ks,
                                   int64_t C, int64_t N, uint32_t width, uint32_t height,
                                   const S* __restrict__ v_means2d,
                                   const S* __restrict__ v_cov2d, S* __restrict__ v_means,
                                   S* __restrict__ v_covars) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    const S px = means[g * 3], py = means[g * 3 + 1], pz = means[g * 3 + 2];
    S cov3[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) cov3[k] = covars[g * 6 + k];
    S acc_p[3] = {0, 0, 0}, acc_s[6] = {0, 0, 0, 0, 0, 0};
    for (int64_t c = 0; c < C; ++c) {
        const View<S> v = load_view(viewmats, Ks, c);
        ProjState<S> p;
        if (!project_state(v, px, py, pz, cov3, static_cast<S>(width), static_cast<S>(height), p))
            continue;
        const int64_t idx = c * N + g;
        S G[6];
#pragma unroll
        for (int k = 0; k < 6; ++k) G[k] = v_cov2d[idx * 6 + k];
        S vp[3], vs[6];
        project_vjp(v, p, v_means2d[idx * 2], v_means2d[idx * 2 + 1], G, vp, vs);
#pragma unroll
        for (int k = 0; k < 3; ++k) acc_p[k] += vp[k];
#pragma unroll
        for (int k = 0; k < 6; ++k) acc_s[k] += vs[k];
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) v_means[g * 3 + k] = acc_p[k];
#pragma unroll
    for (int k = 0; k < 6; ++k) v_covars[g * 6 + k] = acc_s[k];
}

template <typename S>
__global__ void conics_mu_fwd_kernel(const S* __restrict__ cov2d, S eps, S* __restrict__ conics,
                                     S* __restrict__ mus, int64_t total) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    S C[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) C[k] = cov2d[i * 6 + k];
    S u11, u12, u22, mu;
    conic_mu(C, eps, u11, u12, u22, mu);
    conics[i * 3] = u11;
    conics[i * 3 + 1] = u12;
    conics[i * 3 + 2] = u22;
    mus[i] = mu;
}

template <typename S>
__global__ void conics_mu_bwd_kernel(const S* __restrict__ cov2d, S eps,
                                     const S* __restrict__ conics, const S* __restrict__ mus,
                                     const S* __restrict__ v_conics, const S* __restrict__ v_mus,
                                     S* __restrict__ v_cov2d, int64_t total) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    S C[6], g[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) C[k] = cov2d[i * 6 + k];
    conic_mu_vjp(C, eps, conics[i * 3], conics[i * 3 + 1], conics[i * 3 + 2], mus[i],
                 v_conics[i * 3], v_conics[i * 3 + 1], v_conics[i * 3 + 2], v_mus[i], g);
#pragma unroll
    for (int k = 0; k < 6; ++k) v_cov2d[i * 6 + k] = g[k];
}

// ===========================================================================
// World -> volume mapping  (reference: csrc/WorldToVolumeMappingFwd.cu:89-189,
// csrc/WorldToVolumeMappingBwd.cu:82-198)
// ===========================================================================

// Cofactor inverse of a symmetric 3x3 (WorldToVolumeMappingFwd.cu:55-83).
// Expression order fixed.
template <typename S>
__device__ __forceinline__ bool sym3_inverse(const S a[6], S inv[6]) {
    const S a00 = a[0], a01 = a[1], a02 = a[2], a11 = a[3], a12 = a[4], a22 = a[5];
    const S c00 = a11 * a22 - a12 * a12;
    const S c01 = a02 * a12 - a01 * a22;
    const S c02 = a01 * a12 - a02 * a11;
    const S c11 = a00 * a22 - a02 * a02;
    const S c12 = a01 * a02 - a00 * a12;
    const S c22 = a00 * a11 - a01 * a01;
    const S det = a00 * c00 + a01 * c01 + a02 * c02;
    if (abs(det) < static_cast<S>(1e-12)) {
#pragma unroll
        for (int k = 0; k < 6; ++k) inv[k] = static_cast<S>(0);
        return false;
    }
    const S r = static_cast<S>(1) / det;
    inv[0] = c00 * r;
    inv[1] = c01 * r;
    inv[2] = c02 * r;
    inv[3] = c11 * r;
    inv[4] = c12 * r;
    inv[5] = c22 * r;
    return true;
}

// Voxel-space mean and blurred covariance.  Expression order fixed
// (WorldToVolumeMappingFwd.cu:113-150).
template <typename S>
struct VolMap {
    S r0, r1, r2;
    S m[3];
    S Sv[6];
};

template <typename S>
__device__ __forceinline__ void vol_map(const S* __restrict__ p, const S* __restrict__ cov,
                                        const S* __restrict__ ranges,
                                        const S* __restrict__ centers, uint32_t dim2,
                                        uint32_t dim1, uint32_t dim0, S eps3d, VolMap<S>& o) {
    const S D2 = static_cast<S>(dim2), D1 = static_cast<S>(dim1), D0 = static_cast<S>(dim0);
    o.r0 = D2 / ranges[0];
    o.r1 = D1 / ranges[1];
    o.r2 = D0 / ranges[2];
    o.m[0] = (p[0] - centers[0]) * o.r0 + D2 * static_cast<S>(0.5);
    o.m[1] = (p[1] - centers[1]) * o.r1 + D1 * static_cast<S>(0.5);
    o.m[2] = (p[2] - centers[2]) * o.r2 + D0 * static_cast<S>(0.5);
    o.Sv[0] = o.r0 * o.r0 * cov[0];
    o.Sv[1] = o.r0 * o.r1 * cov[1];
    o.Sv[2] = o.r0 * o.r2 * cov[2];
    o.Sv[3] = o.r1 * o.r1 * cov[3];
    o.Sv[4] = o.r1 * o.r2 * cov[4];
    o.Sv[5] = o.r2 * o.r2 * cov[5];
    o.Sv[0] += eps3d;
    o.Sv[3] += eps3d;
    o.Sv[5] += eps3d;
}

// Radii from the blurred voxel covariance (WorldToVolumeMappingFwd.cu:168-188).
template <typename S>
__device__ __forceinline__ bool vol_radii(const S Sv[6], S clip, int32_t r[3]) {
    const S rx = ceil(clip * sqrt(max(static_cast<S>(0), Sv[0])));
    const S ry = ceil(clip * sqrt(max(static_cast<S>(0), Sv[3])));
    const S rz = ceil(clip * sqrt(max(static_cast<S>(0), Sv[5])));
    r[0] = r[1] = r[2] = 0;
    if (!isfinite(rx) || !isfinite(ry) || !isfinite(rz) || rx <= static_cast<S>(0) ||
        ry <= static_cast<S>(0) || rz <= static_cast<S>(0))
        return false;
    r[0] = static_cast<int32_t>(rx);
    r[1] = static_cast<int32_t>(ry);
    r[2] = static_cast<int32_t>(rz);
    return true;
}

// VJP of the mapping given the voxel-space cotangents
// (WorldToVolumeMappingBwd.cu:104-197): v_means = v_m * r;
// v_cov = sym(-P Vu P) scaled by r_i r_j, with Vu the upper-triangular
// cotangent of the stored conic entries.
template <typename S>
__device__ __forceinline__ void vol_map_vjp(const VolMap<S>& o, const S vm[3], const S vc[6],
                                            S v_p[3], S v_cov[6]) {
    v_p[0] = vm[0] * o.r0;
    v_p[1] = vm[1] * o.r1;
    v_p[2] = vm[2] * o.r2;
    S P[6];
    if (!sym3_inverse(o.Sv, P)) {
#pragma unroll
        for (int k = 0; k < 6; ++k) v_cov[k] = static_cast<S>(0);
        return;
    }
    const S P00 = P[0], P01 = P[1], P02 = P[2], P11 = P[3], P12 = P[4], P22 = P[5];
    const S T00 = vc[0] * P00 + vc[1] * P01 + vc[2] * P02;
    const S T01 = vc[0] * P01 + vc[1] * P11 + vc[2] * P12;
    const S T02 = vc[0] * P02 + vc[1] * P12 + vc[2] * P22;
    const S T10 = vc[3] * P01 + vc[4] * P02;
    const S T11 = vc[3] * P11 + vc[4] * P12;
    const S T12 = vc[3] * P12 + vc[4] * P22;
    const S T20 = vc[5] * P02;
    const S T21 = vc[5] * P12;
    const S T22 = vc[5] * P22;
    const S w00 = -(P00 * T00 + P01 * T10 + P02 * T20);
    const S w01 = -(P00 * T01 + P01 * T11 + P02 * T21);
    const S w02 = -(P00 * T02 + P01 * T12 + P02 * T22);
    const S w10 = -(P01 * T00 + P11 * T10 + P12 * T20);
    const S w11 = -(P01 * T01 + P11 * T11 + P12 * T21);
    const S w12 = -(P01 * T02 + P11 * T12 + P12 * T22);
    const S w20 = -(P02 * T00 + P12 * T10 + P22 * T20);
    const S w21 = -(P02 * T01 + P12 * T11 + P22 * T21);
    const S w22 = -(P02 * T02 + P12 * T12 + P22 * T22);
    v_cov[0] = w00 * o.r0 * o.r0;
    v_cov[1] = (w01 + w10) * o.r0 * o.r1;
    v_cov[2] = (w02 + w20) * o.r0 * o.r2;
    v_cov[3] = w11 * o.r1 * o.r1;
    v_cov[4] = (w12 + w21) * o.r1 * o.r2;
    v_cov[5] = w22 * o.r2 * o.r2;
}

template <typename S>
__global__ void map_fwd_kernel(const S* __restrict__ means, const S* __restrict__ covars,
                               const S* __restrict__ ranges, const S* __restrict__ centers,
                               int64_t N, uint32_t dim2, uint32_t dim1, uint32_t dim0, S eps3d,
                               S clip, S* __restrict__ means3d, S* __restrict__ conics,
                               int32_t* __restrict__ radii) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    VolMap<S> o;
    vol_map(means + g * 3, covars + g * 6, ranges, centers, dim2, dim1, dim0, eps3d, o);
#pragma unroll
    for (int k = 0; k < 3; ++k) means3d[g * 3 + k] = o.m[k];
    S P[6];
    const bool ok = sym3_inverse(o.Sv, P);
#pragma unroll
    for (int k = 0; k < 6; ++k) conics[g * 6 + k] = P[k];
    int32_t r[3] = {0, 0, 0};
    if (ok) vol_radii(o.Sv, clip, r);
#pragma unroll
    for (int k = 0; k < 3; ++k) radii[g * 3 + k] = r[k];
}

template <typename S>
__global__ void map_bwd_kernel(const S* __restrict__ means, const S* __restrict__ covars,
                               const S* __restrict__ ranges, const S* __restrict__ centers,
                               int64_t N, uint32_t dim2, uint32_t dim1, uint32_t dim0, S eps3d,
                               const S* __restrict__ v_means3d, const S* __restrict__ v_conics,
                               S* __restrict__ v_means, S* __restrict__ v_covars) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    VolMap<S> o;
    vol_map(means + g * 3, covars + g * 6, ranges, centers, dim2, dim1, dim0, eps3d, o);
    S vm[3], vc[6], vp[3], vcov[6];
#pragma unroll
    for (int k = 0; k < 3; ++k) vm[k] = v_means3d[g * 3 + k];
#pragma unroll
    for (int k = 0; k < 6; ++k) vc[k] = v_conics[g * 6 + k];
    vol_map_vjp(o, vm, vc, vp, vcov);
#pragma unroll
    for (int k = 0; k < 3; ++k) v_means[g * 3 + k] = vp[k];
#pragma unroll
    for (int k = 0; k < 6; ++k) v_covars[g * 6 + k] = vcov[k];
}

// ===========================================================================
// Fused float32 producers of splat records
// ===========================================================================

// Half-extent of the region where w*exp(-q/2...) can reach `thresh`:
// q = d^T Sigma^-1 d / 2 <= s_cut along one axis needs |d_i| <= sqrt(2 s_cut
// Sigma_ii).  The margins cover the float rounding of the conic, of sigma in
// the reference kernels and of __expf; `cond` >= 1 is the conditioning of
// the covariance (the conic's rounding error grows with it).
__device__ __forceinline__ float cull_extent(float s_cut, float sigma_ii, float cond) {
    const float rel = 1.0f + 1e-4f + 4e-7f * cond;
    return sqrtf(2.0f * s_cut * sigma_ii * rel) * 1.0001f + 1e-3f;
}

__device__ __forceinline__ float cull_level(float amp, float thresh) {
    // largest sigma that can still give |amp| * exp(-sigma) >= thresh, widened
    const float a = fabsf(amp);
    if (!(a >= thresh)) return -1.0f;  // also false for NaN
    const float s = logf(a / thresh);
    return s * 1.0001f + 1e-4f;
}

__global__ void project_splats_kernel(const float* __restrict__ means,
                                      const float* __restrict__ covars,
                                      const float* __restrict__ opac,
                                      const float* __restrict__ viewmats,
                                      const float* __restrict__ Ks, int64_t C, int64_t N,
                                      uint32_t width, uint32_t height, uint32_t tile,
                                      uint32_t ntx, uint32_t nty, float eps, float clip,
                                      float* __restrict__ means2d, int32_t* __restrict__ radii,
                                      float4* __restrict__ splats, Rect2* __restrict__ rects,
                                      int32_t* __restrict__ tiles_per_gauss) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= C * N) return;
    const int64_t c = idx / N, g = idx - c * N;
    const View<float> v = load_view(viewmats, Ks, c);
    ProjState<float> p;
    float mx = 0.f, my = 0.f;
    int32_t rx = 0, ry = 0;
    float u11 = 0.f, u12 = 0.f, u22 = 0.f, mu = 0.f;
    float ex = -1.f, ey = -1.f;
    const float w = opac[g];
    if (project_state(v, means[g * 3], means[g * 3 + 1], means[g * 3 + 2], covars + g * 6,
                      static_cast<float>(width), static_cast<float>(height), p)) {
        mx = p.mx;
        my = p.my;
        image_radii(p.C, mx, my, eps, clip, width, height, rx, ry);
        if (conic_mu(p.C, eps, u11, u12, u22, mu)) {
            const float s_cut = cull_level(w * mu, 1e-5f);
            if (s_cut >= 0.0f) {
                const float ab = p.C[0] + eps, db = p.C[3] + eps;
                const float det = ab * db - p.C[1] * p.C[1];
                const float cond = (ab * db) / det;
                if (ab > 0.f && db > 0.f && det > 0.f && isfinite(cond)) {
                    ex = cull_extent(s_cut, ab, cond);
                    ey = cull_extent(s_cut, db, cond);
                } else {
                    ex = ey = CUDART_INF_F;
                }
            }
        }
    }
    means2d[idx * 2] = mx;
    means2d[idx * 2 + 1] = my;
    radii[idx * 2] = rx;
    radii[idx * 2 + 1] = ry;
    splats[idx * 2] = make_float4(mx, my, u11, u12);
    splats[idx * 2 + 1] = make_float4(u22, w * mu, ex, ey);
    int32_t count;
    rects[idx] = tile_rect_2d(mx, my, static_cast<float>(rx), static_cast<float>(ry), tile, ntx,
                              nty, count);
    if (tiles_per_gauss) tiles_per_gauss[idx] = count;
}

__global__ void map_vsplats_kernel(const float* __restrict__ means,
                                   const float* __restrict__ covars,
                                   const float* __restrict__ opac,
                                   const float* __restrict__ ranges,
                                   const float* __restrict__ centers, int64_t N, uint32_t dim2,
                                   uint32_t dim1, uint32_t dim0, uint32_t tile, uint32_t nt2,
                                   uint32_t nt1, uint32_t nt0, float eps3d, float clip,
                                   float* __restrict__ means3d, float* __restrict__ conics,
                                   int32_t* __restrict__ radii, float4* __restrict__ vsplats,
                                   Rect3* __restrict__ rects, int32_t* __restrict__ tiles_per_gauss) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    VolMap<float> o;
    vol_map(means + g * 3, covars + g * 6, ranges, centers, dim2, dim1, dim0, eps3d, o);
    float P[6];
    const bool ok = sym3_inverse(o.Sv, P);
    int32_t r[3] = {0, 0, 0};
    if (ok) vol_radii(o.Sv, clip, r);
#pragma unroll
    for (int k = 0; k < 3; ++k) means3d[g * 3 + k] = o.m[k];
#pragma unroll
    for (int k = 0; k < 6; ++k) conics[g * 6 + k] = P[k];
#pragma unroll
    for (int k = 0; k < 3; ++k) radii[g * 3 + k] = r[k];
    const float w = opac[g];
    float e[3] = {-1.f, -1.f, -1.f};
    if (ok) {
        const float s_cut = cull_level(w, 1e-6f);
        if (s_cut >= 0.0f) {
            const float* A = o.Sv;
            const float det = A[0] * (A[3] * A[5] - A[4] * A[4]) - A[1] * (A[1] * A[5] - A[4] * A[2]) +
                              A[2] * (A[1] * A[4] - A[3] * A[2]);
            const float cond = (A[0] * A[3] * A[5]) / det;
            if (A[0] > 0.f && A[3] > 0.f && A[5] > 0.f && det > 0.f && isfinite(cond)) {
                e[0] = cull_extent(s_cut, A[0], cond);
                e[1] = cull_extent(s_cut, A[3], cond);
                e[2] = cull_extent(s_cut, A[5], cond);
            } else {
                e[0] = e[1] = e[2] = CUDART_INF_F;
            }
        }
    }
    float4* out = vsplats + g * 4;
    out[0] = make_float4(o.m[0], o.m[1], o.m[2], P[0]);
    out[1] = make_float4(P[1], P[2], P[3], P[4]);
    out[2] = make_float4(P[5], w, e[0], e[1]);
    // the voxel backward's cut-off band (r2s_cutoff.cuh)
    out[3] = make_float4(e[2], cutoff_band_v(P, s_threshold_v(w), e[0], e[1], e[2]), 0.f, 0.f);
    int32_t count;
    rects[g] = tile_rect_3d(o.m[0], o.m[1], o.m[2], static_cast<float>(r[0]),
                            static_cast<float>(r[1]), static_cast<float>(r[2]), tile, nt2, nt1,
                            nt0, count);
    if (tiles_per_gauss) tiles_per_gauss[g] = count;
}

// ===========================================================================
// Fused explicit backward (float32), one thread per Gaussian
// ===========================================================================

// Densification statistics of BinaryTreeStrategy._update_state
// (src/strategies/binary_tree.py:305-347, unpacked renders) taken from the
// per-view screen-space gradients as the explicit backward produces them.
struct DensifyArgs {
    const int2* radii;  // [C,N,2]; a view counts when max(rx, ry) > 0
    float scale_x, scale_y, extent;
    int absgrad;       // 1: v_means2d_abs, 0: v_means2d
    float* grad2d;     // [N] += |(g_x scale_x, g_y scale_y)| per counted view; NULL: off
    float* count;      // [N] += counted views
    float* max_radii;  // [N] max(.., max radius / extent) when non-NULL
};

__global__ void explicit_bwd_kernel(
    const float* __restrict__ means, const float* __restrict__ quats,
    const float* __restrict__ raw_scales, const float* __restrict__ raw_opac, float smin,
    float smax, const float* __restrict__ viewmats, const float* __restrict__ Ks, int64_t C,
    int64_t N, uint32_t width, uint32_t height, float eps2d,
    const float4* __restrict__ rstats, float2* __restrict__ v_means2d,
    float2* __restrict__ v_means2d_abs, const float* __restrict__ ranges,
    const float* __restrict__ centers, uint32_t dim2, uint32_t dim1, uint32_t dim0, float eps3d,
    const double* __restrict__ vstats, int accumulate, float* __restrict__ out_means,
    float* __restrict__ out_quats, float* __restrict__ out_scales,
    float* __restrict__ out_opac, DensifyArgs dens) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    RotScale<float> rs;
    rot_scale(quats + g * 4, raw_scales + g * 3, smin, smax, rs);
    float cov3[6];
    covar_from(rs, cov3);
    const float w = softplus_f(raw_opac[g]);
    const float px = means[g * 3], py = means[g * 3 + 1], pz = means[g * 3 + 2];

    float acc_p[3] = {0.f, 0.f, 0.f}, acc_s[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float acc_w = 0.f;
    // densification sums, in the operation order of densify_stats_kernel
    float d_acc = 0.f, d_cnt = 0.f, d_rmax = 0.f;
    if (rstats != nullptr || dens.grad2d != nullptr) {
        for (int64_t c = 0; c < C; ++c) {
            const int64_t idx = c * N + g;
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 s0 = rstats != nullptr ? rstats[idx * 2] : zero;
            const float4 s1 = rstats != nullptr ? rstats[idx * 2 + 1] : zero;
            const View<float> v = load_view(viewmats, Ks, c);
            ProjState<float> p;
            float vmx = 0.f, vmy = 0.f, amx = 0.f, amy = 0.f;
            const bool front = project_state(v, px, py, pz, cov3, static_cast<float>(width),
                                             static_cast<float>(height), p);
            const bool any = (s0.x != 0.f) | (s0.y != 0.f) | (s0.z != 0.f) | (s0.w != 0.f) |
                             (s1.x != 0.f) | (s1.y != 0.f);
            if (front && any) {
                float u11, u12, u22, mu;
                conic_mu(p.C, eps2d, u11, u12, u22, mu);
                const float wm = w * mu;
                // per-view cotangents of the rasterizer inputs
                vmx = wm * (u11 * s0.y + u12 * s0.z);
                vmy = wm * (u12 * s0.y + u22 * s0.z);
                amx = fabsf(wm) * s1.z;
                amy = fabsf(wm) * s1.w;
                const float vu11 = -wm * 0.5f * s0.w;
                const float vu12 = -wm * s1.x;
                const float vu22 = -wm * 0.5f * s1.y;
                const float vmu = w * s0.x;
                acc_w += mu * s0.x;
                float G[6], vp[3], vs[6];
                conic_mu_vjp(p.C, eps2d, u11, u12, u22, mu, vu11, vu12, vu22, vmu, G);
                project_vjp(v, p, vmx, vmy, G, vp, vs);
#pragma unroll
                for (int k = 0; k < 3; ++k) acc_p[k] += vp[k];
#pragma unroll
                for (int k = 0; k < 6; ++k) acc_s[k] += vs[k];
            } else if (front) {
                // mean-gradient only through the projection of means2d (zero here)
            }
            if (v_means2d) v_means2d[idx] = make_float2(vmx, vmy);
            if (v_means2d_abs) v_means2d_abs[idx] = make_float2(amx, amy);
            if (dens.grad2d != nullptr) {
                const int2 r2 = dens.radii[idx];
                const int32_t r = max(r2.x, r2.y);
                if (r > 0) {
                    const float x = __fmul_rn(dens.absgrad ? amx : vmx, dens.scale_x);
                    const float y = __fmul_rn(dens.absgrad ? amy : vmy, dens.scale_y);
                    d_acc = __fadd_rn(d_acc, __fsqrt_rn(__fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y))));
                    d_cnt = __fadd_rn(d_cnt, 1.f);
                    d_rmax = fmaxf(d_rmax, __fdiv_rn((float)r, dens.extent));
                }
            }
        }
    }
    if (dens.grad2d != nullptr) {
        dens.grad2d[g] = __fadd_rn(dens.grad2d[g], d_acc);
        dens.count[g] = __fadd_rn(dens.count[g], d_cnt);
        if (dens.max_radii != nullptr && d_cnt > 0.f)
            dens.max_radii[g] = fmaxf(dens.max_radii[g], d_rmax);
    }
    if (vstats != nullptr) {
        // float64 sums (S0, Sx, Sy, Sz | Sxx, Sxy, Sxz, Syy | Syz, Szz, -, -), each
        // rounded once to float
        const double* vs = vstats + g * 12;
        const float4 t0 = make_float4((float)vs[0], (float)vs[1], (float)vs[2], (float)vs[3]);
        const float4 t1 = make_float4((float)vs[4], (float)vs[5], (float)vs[6], (float)vs[7]);
        const float4 t2 = make_float4((float)vs[8], (float)vs[9], 0.f, 0.f);
        VolMap<float> o;
        vol_map(means + g * 3, cov3, ranges, centers, dim2, dim1, dim0, eps3d, o);
        float P[6];
        if (sym3_inverse(o.Sv, P)) {
            const float vm[3] = {w * (P[0] * t0.y + P[1] * t0.z + P[2] * t0.w),
                                 w * (P[1] * t0.y + P[3] * t0.z + P[4] * t0.w),
                                 w * (P[2] * t0.y + P[4] * t0.z + P[5] * t0.w)};
            const float vc[6] = {-w * 0.5f * t1.x, -w * t1.y, -w * t1.z,
                                 -w * 0.5f * t1.w, -w * t2.x, -w * 0.5f * t2.y};
            float vp[3], vcov[6];
            vol_map_vjp(o, vm, vc, vp, vcov);
#pragma unroll
            for (int k = 0; k < 3; ++k) acc_p[k] += vp[k];
#pragma unroll
            for (int k = 0; k < 6; ++k) acc_s[k] += vcov[k];
        }
        acc_w += t0.x;
    }
    float vq[4], vso[3];
    covar_vjp(rs, acc_s, smin, smax, vq, vso);
    const float vop = acc_w * sigmoid_f(raw_opac[g]);
    if (accumulate) {
#pragma unroll
        for (int k = 0; k < 3; ++k) out_means[g * 3 + k] += acc_p[k];
#pragma unroll
        for (int k = 0; k < 4; ++k) out_quats[g * 4 + k] += vq[k];
#pragma unroll
        for (int k = 0; k < 3; ++k) out_scales[g * 3 + k] += vso[k];
        out_opac[g] += vop;
    } else {
#pragma unroll
        for (int k = 0; k < 3; ++k) out_means[g * 3 + k] = acc_p[k];
#pragma unroll
        for (int k = 0; k < 4; ++k) out_quats[g * 4 + k] = vq[k];
#pragma unroll
        for (int k = 0; k < 3; ++k) out_scales[g * 3 + k] = vso[k];
        out_opac[g] = vop;
    }
}

}  // namespace r2s

// ===========================================================================
// C ABI
// ===========================================================================
using namespace r2s;

extern "C" int r2s_parameter_transform_fwd(int dtype, const void* quats, const void* raw_scales,
                                           double smin, double smax, void* covars,
                                           void* max_scales, int64_t n, r2s_stream_t stream) {
    R2S_REQUIRE(n >= 0, "parameter_transform_fwd: negative N");
    if (n == 0) return R2S_OK;
    return R2S_DTYPE_DISPATCH(dtype, "parameter_transform_fwd", [&] {
        param_fwd_kernel<scalar_t><<<grid_for(n), kThreads, 0, stream>>>(
            (const scalar_t*)quats, (const scalar_t*)raw_scales, (scalar_t)smin, (scalar_t)smax,
            (scalar_t*)covars, (scalar_t*)max_scales, n);
        return check_launch("parameter_transform_fwd");
    });
}

extern "C" int r2s_parameter_transform_bwd(int dtype, const void* quats, const void* raw_scales,
                                           double smin, double smax, const void* v_covars,
                                           void* v_quats, void* v_raw_scales, int64_t n,
                                           r2s_stream_t stream) {
    R2S_REQUIRE(n >= 0, "parameter_transform_bwd: negative N");
    if (n == 0) return R2S_OK;
    return R2S_DTYPE_DISPATCH(dtype, "parameter_transform_bwd", [&] {
        param_bwd_kernel<scalar_t><<<grid_for(n), kThreads, 0, stream>>>(
            (const scalar_t*)quats, (const scalar_t*)raw_scales, (scalar_t)smin, (scalar_t)smax,
            (const scalar_t*)v_covars, (scalar_t*)v_quats, (scalar_t*)v_raw_scales, n);
        return check_launch("parameter_transform_bwd");
    });
}

extern "C" int r2s_prepare_gaussians_f32(const float* quats, const float* raw_scales,
                                         const float* raw_opacities, double smin, double smax,
                                         float* covars, float* max_scales, float* opacities,
                                         int64_t n, r2s_stream_t stream) {
    R2S_REQUIRE(n >= 0, "prepare_gaussians: negative N");
    if (n == 0) return R2S_OK;
    prepare_kernel<<<grid_for(n), kThreads, 0, stream>>>(quats, raw_scales, (float)smin,
                                                          (float)smax, covars, max_scales, n);
    if (int rc = check_launch("prepare_gaussians")) return rc;
    return launch_softplus_f32(raw_opacities, opacities, n, stream);
}

extern "C" int r2s_world_to_image_projection_fwd(int dtype, const void* means, const void* covars,
                                                 const void* viewmats, const void* Ks, int64_t C,
                                                 int64_t N, uint32_t width, uint32_t height,
                                                 double eps2d, double clip, void* means2d,
                                                 void* cov2d, int32_t* radii,
                                                 r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "world_to_image_projection_fwd: negative size");
    R2S_REQUIRE(clip > 0.0, "radius_clip must be positive");
    if (C * N == 0) return R2S_OK;
    R2S_REQUIRE(C * N < (int64_t(1) << 31) * 32, "world_to_image_projection_fwd: C*N too large");
    return R2S_DTYPE_DISPATCH(dtype, "world_to_image_projection_fwd", [&] {
        project_fwd_kernel<scalar_t><<<grid_for(C * N), kThreads, 0, stream>>>(
            (const scalar_t*)means, (const scalar_t*)covars, (const scalar_t*)viewmats,
            (const scalar_t*)Ks, C, N, width, height, (scalar_t)eps2d, (scalar_t)clip,
            (scalar_t*)means2d, (scalar_t*)cov2d, radii);
        return check_launch("world_to_image_projection_fwd");
    });
}

extern "C" int r2s_world_to_image_projection_bwd(int dtype, const void* means, const void* covars,
                                                 const void* viewmats, const void* Ks, int64_t C,
                                                 int64_t N, uint32_t width, uint32_t height,
                                                 const void* v_means2d, const void* v_cov2d,
                                                 void* v_means, void* v_covars,
                                                 r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "world_to_image_projection_bwd: negative size");
    if (N == 0) return R2S_OK;
    if (C == 0) {
        const size_t es = dtype == R2S_F64 ? 8 : 4;
        cudaMemsetAsync(v_means, 0, N * 3 * es, stream);
        cudaMemsetAsync(v_covars, 0, N * 6 * es, stream);
        return check_launch("world_to_image_projection_bwd");
    }
    return R2S_DTYPE_DISPATCH(dtype, "world_to_image_projection_bwd", [&] {
        project_bwd_kernel<scalar_t><<<grid_for(N, 128), 128, 0, stream>>>(
            (const scalar_t*)means, (const scalar_t*)covars, (const scalar_t*)viewmats,
            (const scalar_t*)Ks, C, N, width, height, (const scalar_t*)v_means2d,
            (const scalar_t*)v_cov2d, (scalar_t*)v_means, (scalar_t*)v_covars);
        return check_launch("world_to_image_projection_bwd");
    });
}

extern "C" int r2s_conics_mu_fwd(int dtype, const void* cov2d, double eps, void* conics, void* mus,
                                 int64_t total, r2s_stream_t stream) {
    R2S_REQUIRE(total >= 0, "conics_mu_fwd: negative size");
    if (total == 0) return R2S_OK;
    return R2S_DTYPE_DISPATCH(dtype, "conics_mu_fwd", [&] {
        conics_mu_fwd_kernel<scalar_t><<<grid_for(total), kThreads, 0, stream>>>(
            (const scalar_t*)cov2d, (scalar_t)eps, (scalar_t*)conics, (scalar_t*)mus, total);
        return check_launch("conics_mu_fwd");
    });
}

extern "C" int r2s_conics_mu_bwd(int dtype, const void* cov2d, double eps, const void* conics,
                                 const void* mus, const void* v_conics, const void* v_mus,
                                 void* v_cov2d, int64_t total, r2s_stream_t stream) {
    R2S_REQUIRE(total >= 0, "conics_mu_bwd: negative size");
    if (total == 0) return R2S_OK;
    return R2S_DTYPE_DISPATCH(dtype, "conics_mu_bwd", [&] {
        conics_mu_bwd_kernel<scalar_t><<<grid_for(total), kThreads, 0, stream>>>(
            (const scalar_t*)cov2d, (scalar_t)eps, (const scalar_t*)conics,
            (const scalar_t*)mus, (const scalar_t*)v_conics, (const scalar_t*)v_mus,
            (scalar_t*)v_cov2d, total);
        return check_launch("conics_mu_bwd");
    });
}

extern "C" int r2s_world_to_volume_mapping_fwd(int dtype, const void* means, const void* covars,
                                               const void* max_scales, const void* ranges,
                                               const void* centers, int64_t N, uint32_t dim2,
                                               uint32_t dim1, uint32_t dim0, double eps3d,
                                               double clip, void* means3d, void* conics,
                                               int32_t* radii, r2s_stream_t stream) {
    (void)max_scales;
    R2S_REQUIRE(N >= 0, "world_to_volume_mapping_fwd: negative N");
    if (N == 0) return R2S_OK;
    return R2S_DTYPE_DISPATCH(dtype, "world_to_volume_mapping_fwd", [&] {
        map_fwd_kernel<scalar_t><<<grid_for(N), kThreads, 0, stream>>>(
            (const scalar_t*)means, (const scalar_t*)covars, (const scalar_t*)ranges,
            (const scalar_t*)centers, N, dim2, dim1, dim0, (scalar_t)eps3d, (scalar_t)clip,
            (scalar_t*)means3d, (scalar_t*)conics, radii);
        return check_launch("world_to_volume_mapping_fwd");
    });
}

extern "C" int r2s_world_to_volume_mapping_bwd(int dtype, const void* means, const void* covars,
                                               const void* ranges, const void* centers, int64_t N,
                                               uint32_t dim2, uint32_t dim1, uint32_t dim0,
                                               double eps3d, const void* v_means3d,
                                               const void* v_conics, void* v_means,
                                               void* v_covars, r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0, "world_to_volume_mapping_bwd: negative N");
    if (N == 0) return R2S_OK;
    return R2S_DTYPE_DISPATCH(dtype, "world_to_volume_mapping_bwd", [&] {
        map_bwd_kernel<scalar_t><<<grid_for(N), kThreads, 0, stream>>>(
            (const scalar_t*)means, (const scalar_t*)covars, (const scalar_t*)ranges,
            (const scalar_t*)centers, N, dim2, dim1, dim0, (scalar_t)eps3d,
            (const scalar_t*)v_means3d, (const scalar_t*)v_conics, (scalar_t*)v_means,
            (scalar_t*)v_covars);
        return check_launch("world_to_volume_mapping_bwd");
    });
}

extern "C" int r2s_project_splats_f32(const float* means, const float* covars,
                                      const float* opacities, const float* viewmats,
                                      const float* Ks, int64_t C, int64_t N, uint32_t width,
                                      uint32_t height, uint32_t tile, uint32_t ntx, uint32_t nty,
                                      double eps2d, double clip, float* means2d, int32_t* radii,
                                      float* splats, void* rects, int32_t* tiles_per_gauss,
                                      r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "project_splats: negative size");
    R2S_REQUIRE(clip > 0.0, "radius_clip must be positive");
    R2S_REQUIRE(tile > 0, "tile_size must be positive");
    R2S_REQUIRE(ntx < 65536 && nty < 65536, "project_splats: tile grid too large");
    if (C * N == 0) return R2S_OK;
    project_splats_kernel<<<grid_for(C * N), kThreads, 0, stream>>>(
        means, covars, opacities, viewmats, Ks, C, N, width, height, tile, ntx, nty,
        (float)eps2d, (float)clip, means2d, radii, (float4*)splats, (Rect2*)rects,
        tiles_per_gauss);
    return check_launch("project_splats");
}

extern "C" int r2s_map_vsplats_f32(const float* means, const float* covars, const float* opacities,
                                   const float* ranges, const float* centers, int64_t N,
                                   uint32_t dim2, uint32_t dim1, uint32_t dim0, uint32_t tile,
                                   uint32_t nt2, uint32_t nt1, uint32_t nt0, double eps3d,
                                   double clip, float* means3d, float* conics, int32_t* radii,
                                   float* vsplats, void* rects3, int32_t* tiles_per_gauss,
                                   r2s_stream_t stream) {
    R2S_REQUIRE(N >= 0, "map_vsplats: negative N");
    R2S_REQUIRE(tile > 0, "tile_size must be positive");
    R2S_REQUIRE(nt0 < 65536 && nt1 < 65536 && nt2 < 65536, "map_vsplats: brick grid too large");
    if (N == 0) return R2S_OK;
    map_vsplats_kernel<<<grid_for(N), kThreads, 0, stream>>>(
        means, covars, opacities, ranges, centers, N, dim2, dim1, dim0, tile, nt2, nt1, nt0,
        (float)eps3d, (float)clip, means3d, conics, radii, (float4*)vsplats, (Rect3*)rects3,
        tiles_per_gauss);
    return check_launch("map_vsplats");
}

namespace {
int explicit_backward_launch(
    const float* means, const float* quats, const float* raw_scales, const float* raw_opacities,
    double smin, double smax, const float* viewmats, const float* Ks, int64_t C, int64_t N,
    uint32_t width, uint32_t height, double eps2d, const float* raster_stats, float* v_means2d,
    float* v_means2d_abs, const float* ranges, const float* centers, uint32_t dim2,
    uint32_t dim1, uint32_t dim0, double eps3d, const double* vox_stats, int accumulate,
    float* v_means, float* v_quats, float* v_raw_scales, float* v_raw_opacities,
    const r2s_densify_args* densify, r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "explicit_backward: negative size");
    R2S_REQUIRE(vox_stats == nullptr || (ranges && centers),
                "explicit_backward: voxel statistics need ranges and centers");
    DensifyArgs dens{};
    if (densify != nullptr) {
        R2S_REQUIRE(densify->grad2d && densify->count && (C == 0 || densify->radii),
                    "explicit_backward: densify statistics need radii, grad2d and count");
        R2S_REQUIRE(densify->extent > 0.0, "explicit_backward: densify extent must be positive");
        R2S_REQUIRE(C == 0 || viewmats, "explicit_backward: densify statistics need the views");
        dens.radii = reinterpret_cast<const int2*>(densify->radii);
        dens.scale_x = (float)densify->scale_x;
        dens.scale_y = (float)densify->scale_y;
        dens.extent = (float)densify->extent;
        dens.absgrad = densify->absgrad ? 1 : 0;
        dens.grad2d = densify->grad2d;
        dens.count = densify->count;
        dens.max_radii = densify->max_radii;
    }
    if (N == 0) return R2S_OK;
    explicit_bwd_kernel<<<grid_for(N, 128), 128, 0, stream>>>(
        means, quats, raw_scales, raw_opacities, (float)smin, (float)smax, viewmats, Ks, C, N,
        width, height, (float)eps2d, (const float4*)raster_stats, (float2*)v_means2d,
        (float2*)v_means2d_abs, ranges, centers, dim2, dim1, dim0, (float)eps3d,
        vox_stats, accumulate, v_means, v_quats, v_raw_scales, v_raw_opacities,
        dens);
    return check_launch("explicit_backward");
}
}  // namespace

extern "C" int r2s_explicit_backward_f32(
    const float* means, const float* quats, const float* raw_scales, const float* raw_opacities,
    double smin, double smax, const float* viewmats, const float* Ks, int64_t C, int64_t N,
    uint32_t width, uint32_t height, double eps2d, const float* raster_stats, float* v_means2d,
    float* v_means2d_abs, const float* ranges, const float* centers, uint32_t dim2,
    uint32_t dim1, uint32_t dim0, double eps3d, const double* vox_stats, int accumulate,
    float* v_means, float* v_quats, float* v_raw_scales, float* v_raw_opacities,
    r2s_stream_t stream) {
    return explicit_backward_launch(means, quats, raw_scales, raw_opacities, smin, smax, viewmats,
                                    Ks, C, N, width, height, eps2d, raster_stats, v_means2d,
                                    v_means2d_abs, ranges, centers, dim2, dim1, dim0, eps3d,
                                    vox_stats, accumulate, v_means, v_quats, v_raw_scales,
                                    v_raw_opacities, nullptr, stream);
}

extern "C" int r2s_explicit_backward_densify_f32(
    const float* means, const float* quats, const float* raw_scales, const float* raw_opacities,
    double smin, double smax, const float* viewmats, const float* Ks, int64_t C, int64_t N,
    uint32_t width, uint32_t height, double eps2d, const float* raster_stats, float* v_means2d,
    float* v_means2d_abs, const float* ranges, const float* centers, uint32_t dim2,
    uint32_t dim1, uint32_t dim0, double eps3d, const double* vox_stats, int accumulate,
    float* v_means, float* v_quats, float* v_raw_scales, float* v_raw_opacities,
    const r2s_densify_args* densify, r2s_stream_t stream) {
    R2S_REQUIRE(densify != nullptr, "explicit_backward_densify: null densify arguments");
    return explicit_backward_launch(means, quats, raw_scales, raw_opacities, smin, smax, viewmats,
                                    Ks, C, N, width, height, eps2d, raster_stats, v_means2d,
                                    v_means2d_abs, ranges, centers, dim2, dim1, dim0, eps3d,
                                    vox_stats, accumulate, v_means, v_quats, v_raw_scales,
                                    v_raw_opacities, densify, stream);
}
