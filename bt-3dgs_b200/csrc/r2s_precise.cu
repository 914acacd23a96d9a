// Elementwise kernels compiled WITHOUT fast math (build.py: files named
// *_precise.cu).
//
// The reference activates the raw opacities with
// torch.nn.functional.softplus(beta=1, threshold=20) (r2splat/ops/direct.py:96)
// in float: x > 20 ? x : log1p(exp(x)), with the CUDA math library's
// accurate expf/log1pf and no flush-to-zero.  Every later cut-off decision of
// the rasterizer and voxelizer (|opacity * mu * exp(-sigma)| >= 1e-5 or
// |opacity * exp(-sigma)| >= 1e-6) compares a product of this value, so the
// opacity is computed here with the same float operations, in a translation
// unit whose expf and log1pf are the accurate ones (a fast-math unit would
// substitute the approximate intrinsics).
#include "r2s_common.cuh"

namespace r2s {
namespace {

__global__ void softplus_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = x[i];
    y[i] = v * 1.0f > 20.0f ? v : log1pf(expf(v * 1.0f)) / 1.0f;
}

}  // namespace

int launch_softplus_f32(const float* x, float* y, int64_t n, cudaStream_t stream) {
    if (n <= 0) return R2S_OK;
    softplus_kernel<<<grid_for(n), kThreads, 0, stream>>>(x, y, n);
    return check_launch("softplus");
}

}  // namespace r2s

// ===========================================================================
// Binary-tree split: the two children of each selected Gaussian
// (reference: split(), src/strategies/binary_tree.py:92-149)
// ===========================================================================
//
// For a selected Gaussian with activated scales s (bounded sigmoid,
// s = lo + (hi - lo) sigmoid(raw), src/models/gaussian_model.py:252-259) and
// rotation R of its normalized quaternion (src/utils/math.py:35-53), the
// longest axis k (first maximum) gives the offset R[:, k] s_k; the children
// sit at mean + offset (first block of S) and mean - offset (second block),
// both with s_k divided by 1.6 (floored at 1e-12) mapped back through the
// inverse activation (clamp to [lo + eps, hi - eps], normalize, clamp to
// [1e-6, 1 - 1e-6], logit: gaussian_model.py:261-270), the parent's raw
// quaternion, and the parent's raw opacity or, with the revised rule,
// softplus^-1(1 - sqrt(1 - min(softplus(raw), 0.9999))).  Every step is one
// float operation with its own rounding, as the reference's elementwise torch
// ops are (explicit _rn intrinsics keep the compiler from fusing them), so the
// longest-axis choice and the values follow the reference's arithmetic.
namespace r2s {
namespace {

__device__ __forceinline__ float torch_sigmoid(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
}

__device__ __forceinline__ float torch_softplus(float x) {
    return x > 20.0f ? x : log1pf(expf(x));
}

__global__ void split_children_kernel(const float* __restrict__ means,
                                      const float* __restrict__ raw_scales,
                                      const float* __restrict__ quats,
                                      const float* __restrict__ raw_opac,
                                      const int64_t* __restrict__ sel, int64_t S, float lo,
                                      float hi, float seps, int revised,
                                      float* __restrict__ c_means, float* __restrict__ c_scales,
                                      float* __restrict__ c_quats, float* __restrict__ c_opac) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S) return;
    const int64_t g = sel[i];
    const float span = __fsub_rn(hi, lo);
    float s[3];
#pragma unroll
    for (int k = 0; k < 3; ++k)
        s[k] = __fadd_rn(lo, __fmul_rn(span, torch_sigmoid(raw_scales[g * 3 + k])));
    int ax = 0;  // first maximum, as torch.argmax
    if (s[1] > s[ax]) ax = 1;
    if (s[2] > s[ax]) ax = 2;

    const float q0 = quats[g * 4], q1 = quats[g * 4 + 1], q2 = quats[g * 4 + 2],
                q3 = quats[g * 4 + 3];
    const float nrm = fmaxf(sqrtf(__fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(q0, q0), __fmul_rn(q1, q1)),
                                                      __fmul_rn(q2, q2)),
                                            __fmul_rn(q3, q3))),
                            1e-12f);
    const float w = __fdiv_rn(q0, nrm), x = __fdiv_rn(q1, nrm), y = __fdiv_rn(q2, nrm),
                z = __fdiv_rn(q3, nrm);
    // column ax of the rotation matrix (rows 0, 1, 2)
    float c0, c1, c2;
    if (ax == 0) {
        c0 = __fsub_rn(1.0f, __fmul_rn(2.0f, __fadd_rn(__fmul_rn(y, y), __fmul_rn(z, z))));
        c1 = __fmul_rn(2.0f, __fadd_rn(__fmul_rn(x, y), __fmul_rn(w, z)));
        c2 = __fmul_rn(2.0f, __fsub_rn(__fmul_rn(x, z), __fmul_rn(w, y)));
    } else if (ax == 1) {
        c0 = __fmul_rn(2.0f, __fsub_rn(__fmul_rn(x, y), __fmul_rn(w, z)));
        c1 = __fsub_rn(1.0f, __fmul_rn(2.0f, __fadd_rn(__fmul_rn(x, x), __fmul_rn(z, z))));
        c2 = __fmul_rn(2.0f, __fadd_rn(__fmul_rn(y, z), __fmul_rn(w, x)));
    } else {
        c0 = __fmul_rn(2.0f, __fadd_rn(__fmul_rn(x, z), __fmul_rn(w, y)));
        c1 = __fmul_rn(2.0f, __fsub_rn(__fmul_rn(y, z), __fmul_rn(w, x)));
        c2 = __fsub_rn(1.0f, __fmul_rn(2.0f, __fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y))));
    }
    const float off[3] = {__fmul_rn(c0, s[ax]), __fmul_rn(c1, s[ax]), __fmul_rn(c2, s[ax])};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float m = means[g * 3 + k];
        c_means[i * 3 + k] = __fadd_rn(m, off[k]);
        c_means[(S + i) * 3 + k] = __fadd_rn(m, -off[k]);
    }

    const float clamp_lo = __fadd_rn(lo, seps), clamp_hi = __fsub_rn(hi, seps);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        float t = s[k];
        if (k == ax) t = fmaxf(__fdiv_rn(s[k], 1.6f), 1e-12f);
        t = fminf(fmaxf(t, clamp_lo), clamp_hi);
        float p = __fdiv_rn(__fsub_rn(t, lo), span);
        p = fminf(fmaxf(p, 1e-6f), 0.999999f);
        const float raw = logf(__fdiv_rn(p, __fsub_rn(1.0f, p)));
        c_scales[i * 3 + k] = raw;
        c_scales[(S + i) * 3 + k] = raw;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        c_quats[i * 4 + k] = quats[g * 4 + k];
        c_quats[(S + i) * 4 + k] = quats[g * 4 + k];
    }
    float o = raw_opac[g];
    if (revised) {
        const float base = fminf(torch_softplus(o), 0.9999f);
        const float nw = __fsub_rn(1.0f, sqrtf(__fsub_rn(1.0f, base)));
        o = logf(expm1f(nw));
    }
    c_opac[i] = o;
    c_opac[S + i] = o;
}

}  // namespace
}  // namespace r2s

extern "C" int r2s_split_children_f32(const float* means, const float* raw_scales,
                                      const float* quats, const float* raw_opacities,
                                      const int64_t* sel, int64_t S, double scale_min,
                                      double scale_max, double scale_eps, int revised_opacity,
                                      float* child_means, float* child_scales,
                                      float* child_quats, float* child_opacities,
                                      r2s_stream_t stream) {
    R2S_REQUIRE(S >= 0, "split_children: negative count");
    R2S_REQUIRE(scale_max > scale_min, "split_children: scale_max must exceed scale_min");
    if (S == 0) return R2S_OK;
    r2s::split_children_kernel<<<r2s::grid_for(S), r2s::kThreads, 0, (cudaStream_t)stream>>>(
        means, raw_scales, quats, raw_opacities, sel, S, (float)scale_min, (float)scale_max,
        (float)scale_eps, revised_opacity, child_means, child_scales, child_quats,
        child_opacities);
    return r2s::check_launch("split_children");
}
