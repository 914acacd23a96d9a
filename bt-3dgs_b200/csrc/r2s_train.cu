// Training-step kernels on the per-Gaussian parameters (the rows after the
// rasterizer backward in a training step).
//
// Adam: one launch updates every parameter group of the model in place with
// torch.optim.Adam's arithmetic (amsgrad off, no weight decay), the way the
// reference builds its optimizers (src/models/gaussian_model.py:514-530: one
// Adam per parameter group, eps 1e-15) and steps them
// (src/trainers/binary_tree.py:204-206).  Per element, in torch's order:
//   m <- m + (1 - b1) (g - m)          (lerp, weight 1 - b1 < 0.5)
//   v <- v b2 + ((1 - b2) g) g         (mul, addcmul)
//   p <- p + (-lr / bc1) (m / (sqrt(v) / sqrt(bc2) + eps))   (addcdiv)
// with bc1 = 1 - b1^t, bc2 = 1 - b2^t evaluated on the host in double, as
// torch does.  Square root and division are IEEE-rounded (this file does not
// rely on the fast-math approximations of the rest of the library).
//
// Densification statistics: the reference strategy's _update_state
// (src/strategies/binary_tree.py:305-347) scales the per-(view, Gaussian)
// screen-space gradient by (W/2 C, H/2 C), keeps the pairs with radius > 0,
// and index-adds the gradient norms and a count per Gaussian (plus the
// largest radius / max(W, H) when scale-based refinement is on).  Here one
// thread per Gaussian walks its views, so the sums need no atomics and are
// deterministic.
#include <algorithm>
#include <cmath>

#include "r2s_common.cuh"

namespace r2s {

namespace {

constexpr int kMaxAdamGroups = 8;

struct AdamLaunch {
    float* p[kMaxAdamGroups];
    const float* g[kMaxAdamGroups];
    float* m[kMaxAdamGroups];
    float* v[kMaxAdamGroups];
    int64_t end[kMaxAdamGroups];  // exclusive prefix end of each group in the joint index space
    float neg_step_size[kMaxAdamGroups];
    float bc2_sqrt[kMaxAdamGroups];
    int n_groups;
    float beta1, beta2, one_minus_beta1, one_minus_beta2, eps;
};

__global__ void adam_kernel(AdamLaunch a, int64_t total) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int k = 0;
        while (k + 1 < a.n_groups && i >= a.end[k]) ++k;
        const int64_t j = i - (k ? a.end[k - 1] : 0);
        const float g = a.g[k][j];
        float m = a.m[k][j];
        float v = a.v[k][j];
        m = __fmaf_rn(a.one_minus_beta1, __fsub_rn(g, m), m);
        v = __fmaf_rn(__fmul_rn(a.one_minus_beta2, g), g, __fmul_rn(v, a.beta2));
        const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.bc2_sqrt[k]), a.eps);
        const float p = a.p[k][j];
        a.p[k][j] = __fmaf_rn(a.neg_step_size[k], __fdiv_rn(m, denom), p);
        a.m[k][j] = m;
        a.v[k][j] = v;
    }
}

__global__ void densify_stats_kernel(const float* __restrict__ grads2d,
                                     const int32_t* __restrict__ radii, int64_t C, int64_t N,
                                     float scale_x, float scale_y, float extent,
                                     float* __restrict__ grad2d, float* __restrict__ count,
                                     float* __restrict__ max_radii) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= N) return;
    float acc = 0.f, cnt = 0.f, rmax = 0.f;
#pragma unroll 4
    for (int64_t c = 0; c < C; ++c) {
        const int64_t i = c * N + g;
        const int32_t r = radii[i];
        if (r <= 0) continue;
        const float2 d = reinterpret_cast<const float2*>(grads2d)[i];
        const float x = __fmul_rn(d.x, scale_x), y = __fmul_rn(d.y, scale_y);
        acc = __fadd_rn(acc, __fsqrt_rn(__fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y))));
        cnt = __fadd_rn(cnt, 1.f);
        rmax = fmaxf(rmax, __fdiv_rn((float)r, extent));
    }
    grad2d[g] = __fadd_rn(grad2d[g], acc);
    count[g] = __fadd_rn(count[g], cnt);
    if (max_radii != nullptr && cnt > 0.f) max_radii[g] = fmaxf(max_radii[g], rmax);
}

}  // namespace

}  // namespace r2s

using namespace r2s;

extern "C" int r2s_adam_step_f32(const r2s_adam_group* groups, int n_groups, double beta1,
                                 double beta2, double eps, r2s_stream_t stream) {
    R2S_REQUIRE(n_groups >= 0 && n_groups <= kMaxAdamGroups,
                "adam_step: 0 to 8 parameter groups per call");
    R2S_REQUIRE(n_groups == 0 || groups != nullptr, "adam_step: null group array");
    R2S_REQUIRE(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0,
                "adam_step: betas must lie in [0, 1)");
    AdamLaunch a{};
    int64_t total = 0;
    int k = 0;
    for (int i = 0; i < n_groups; ++i) {
        const r2s_adam_group& gr = groups[i];
        R2S_REQUIRE(gr.numel >= 0, "adam_step: negative numel");
        R2S_REQUIRE(gr.step >= 1, "adam_step: step must be >= 1 (the count after this update)");
        if (gr.numel == 0) continue;
        R2S_REQUIRE(gr.param && gr.grad && gr.exp_avg && gr.exp_avg_sq, "adam_step: null pointer");
        const double bc1 = 1.0 - std::pow(beta1, (double)gr.step);
        const double bc2 = 1.0 - std::pow(beta2, (double)gr.step);
        a.p[k] = gr.param;
        a.g[k] = gr.grad;
        a.m[k] = gr.exp_avg;
        a.v[k] = gr.exp_avg_sq;
        total += gr.numel;
        a.end[k] = total;
        a.neg_step_size[k] = (float)(-(gr.lr / bc1));
        a.bc2_sqrt[k] = (float)std::sqrt(bc2);
        ++k;
    }
    a.n_groups = k;
    a.beta1 = (float)beta1;
    a.beta2 = (float)beta2;
    a.one_minus_beta1 = (float)(1.0 - beta1);
    a.one_minus_beta2 = (float)(1.0 - beta2);
    a.eps = (float)eps;
    if (total == 0) return R2S_OK;
    const int64_t blocks = std::min<int64_t>((total + kThreads - 1) / kThreads, 148 * 16);
    adam_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(a, total);
    return check_launch("adam_step");
}

extern "C" int r2s_densify_stats_f32(const float* grads2d, const int32_t* radii, int64_t C,
                                     int64_t N, double scale_x, double scale_y, double extent,
                                     float* grad2d, float* count, float* max_radii,
                                     r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && N >= 0, "densify_stats: negative size");
    R2S_REQUIRE(extent > 0.0, "densify_stats: extent must be positive");
    if (N == 0) return R2S_OK;
    R2S_REQUIRE(grad2d && count && (C == 0 || (grads2d && radii)), "densify_stats: null pointer");
    densify_stats_kernel<<<grid_for(N), kThreads, 0, stream>>>(
        grads2d, radii, C, N, (float)scale_x, (float)scale_y, (float)extent, grad2d, count,
        max_radii);
    return check_launch("densify_stats");
}
