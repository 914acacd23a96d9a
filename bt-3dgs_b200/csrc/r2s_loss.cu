// Training-step losses and their gradients, fused.
//
// Projection losses of BinaryTreeLossComputer (src/utils/loss.py:125-172):
//   l1   = mean |x - t|
//   ssim = mean S, S = ((2 m1 m2 + c1)(2 s12 + c2)) / ((m1^2 + m2^2 + c1)(s11 + s22 + c2))
//          with local statistics from an 11x11 Gaussian window (sigma 1.5,
//          zero padding), m = w*x, s11 = w*(x x) - m1^2, s12 = w*(x t) - m1 m2
//          (ssim2d, src/utils/metric.py:36-56)
//   edge = mean mask |x - te|                  (compute_edge_loss, loss.py:22-23)
// One CTA per (image, 32x32 tile) computes the statistics on the tile plus a
// 5-pixel halo from a 10-pixel input halo (separable passes through shared
// memory), the per-pixel partials of S with respect to m1, w*(x x) and
// w*(x t), and correlates them with the window again for the gradient:
//   d mean S / d x_p = (1/M) [ (w*dS/dm1)(p) + 2 x_p (w*dS/de11)(p) + t_p (w*dS/de12)(p) ].
// The window is separable; the reference convolves with the outer product of
// the same float32 1-D weights, so the two differ by rounding only.  The
// window sums, S, its partials and their correlation are evaluated in double
// (sigma^2 = w*(x x) - m^2 cancels in float on smooth images, and so do the
// mean and second-moment paths of the gradient); inputs and outputs are float.
//
// Volume TV (compute_tv_loss, loss.py:10-21): mean absolute forward difference
// along each axis; d/dv = sign of the backward difference minus sign of the
// forward difference, per axis, over the count of differences.
#include <algorithm>
#include <cmath>

#include "r2s_common.cuh"

namespace r2s {

namespace {

constexpr int kR = 5;                // window radius (11 taps)
constexpr int kTO = 32;              // output tile
constexpr int kTS = kTO + 2 * kR;    // statistics region (42)
constexpr int kTI = kTO + 4 * kR;    // input region (52)
constexpr int kLossThreads = 256;
// inputs in float; the window sums in double: sigma^2 = w*(x x) - m^2 cancels
// badly in float on smooth projections, which is most of what a CT detector sees
constexpr size_t kLossSmem =
    sizeof(float) * 2 * kTI * kTI + sizeof(double) * (5 * kTI * kTS + 5 * kTS * kTS);

struct Window11 {
    double g[2 * kR + 1];
};

__device__ __forceinline__ float sgnf(float v) { return (float)((v > 0.f) - (v < 0.f)); }

__device__ __forceinline__ void block_add3(double a, double b, double c, double* sums) {
    a = warp_sum(a);
    b = warp_sum(b);
    c = warp_sum(c);
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(sums, a);
        atomicAdd(sums + 1, b);
        atomicAdd(sums + 2, c);
    }
}

__global__ void __launch_bounds__(kLossThreads)
proj_loss_kernel(const float* __restrict__ x, const float* __restrict__ t,
                 const float* __restrict__ te, const float* __restrict__ mask, int H, int W,
                 Window11 w, double c1, double c2, const float* __restrict__ weights, double inv_m,
                 float* __restrict__ grad, double* __restrict__ sums) {
    extern __shared__ __align__(16) double smd[];
    double* hz = smd;                     // [5][kTI][kTS], later float partials [3][kTS][kTS]
    double* ss = hz + 5 * kTI * kTS;      // [5][kTS][kTS], later float [3][kTS][kTO]
    float* sx = reinterpret_cast<float*>(ss + 5 * kTS * kTS);  // [kTI][kTI]
    float* st = sx + kTI * kTI;           // [kTI][kTI]
    const int tid = threadIdx.x;
    const int X0 = blockIdx.x * kTO, Y0 = blockIdx.y * kTO;
    const int64_t img = (int64_t)blockIdx.z * H * W;

    for (int i = tid; i < kTI * kTI; i += kLossThreads) {
        const int r = i / kTI, c = i - r * kTI;
        const int gy = Y0 - 2 * kR + r, gx = X0 - 2 * kR + c;
        const bool in = gy >= 0 && gy < H && gx >= 0 && gx < W;
        sx[i] = in ? x[img + (int64_t)gy * W + gx] : 0.f;
        st[i] = in ? t[img + (int64_t)gy * W + gx] : 0.f;
    }
    __syncthreads();
    // horizontal pass of x, t, x x, t t, x t
    for (int i = tid; i < kTI * kTS; i += kLossThreads) {
        const int r = i / kTS, c = i - r * kTS;
        const float* px = sx + r * kTI + c;
        const float* pt = st + r * kTI + c;
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0, a4 = 0.0;
#pragma unroll
        for (int k = 0; k < 2 * kR + 1; ++k) {
            const double u = px[k], v = pt[k], g = w.g[k];
            a0 = fma(g, u, a0);
            a1 = fma(g, v, a1);
            a2 = fma(g * u, u, a2);
            a3 = fma(g * v, v, a3);
            a4 = fma(g * u, v, a4);
        }
        hz[i] = a0;
        hz[kTI * kTS + i] = a1;
        hz[2 * kTI * kTS + i] = a2;
        hz[3 * kTI * kTS + i] = a3;
        hz[4 * kTI * kTS + i] = a4;
    }
    __syncthreads();
    // vertical pass -> m1, m2, e11, e22, e12 on the statistics region
    for (int i = tid; i < kTS * kTS; i += kLossThreads) {
        const int r = i / kTS, c = i - r * kTS;
        double a[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
#pragma unroll
        for (int k = 0; k < 2 * kR + 1; ++k) {
            const double g = w.g[k];
#pragma unroll
            for (int q = 0; q < 5; ++q) a[q] = fma(g, hz[q * kTI * kTS + (r + k) * kTS + c], a[q]);
        }
#pragma unroll
        for (int q = 0; q < 5; ++q) ss[q * kTS * kTS + i] = a[q];
    }
    __syncthreads();
    // S and its partials (zero outside the image)
    double s_sum = 0.0;
    double* part = hz;  // [3][kTS][kTS]
    for (int i0 = 0; i0 < kTS * kTS; i0 += kLossThreads) {
        const int i = i0 + tid;
        double p1 = 0.0, p2 = 0.0, p3 = 0.0;
        if (i < kTS * kTS) {
            const int r = i / kTS, c = i - r * kTS;
            const int gy = Y0 - kR + r, gx = X0 - kR + c;
            if (gy >= 0 && gy < H && gx >= 0 && gx < W) {
                const double m1 = ss[i], m2 = ss[kTS * kTS + i];
                const double e11 = ss[2 * kTS * kTS + i], e22 = ss[3 * kTS * kTS + i];
                const double e12 = ss[4 * kTS * kTS + i];
                const double m11 = m1 * m1, m22 = m2 * m2, m12 = m1 * m2;
                const double A1 = 2.0 * m12 + c1;
                const double A2 = 2.0 * (e12 - m12) + c2;
                const double B1 = m11 + m22 + c1;
                const double B2 = (e11 - m11) + (e22 - m22) + c2;
                const double inv_b = 1.0 / (B1 * B2);
                const double S = A1 * A2 * inv_b;
                if (r >= kR && r < kR + kTO && c >= kR && c < kR + kTO) s_sum += S;
                p1 = 2.0 * m2 * (A2 - A1) * inv_b - 2.0 * m1 * S * (1.0 / B1 - 1.0 / B2);
                p2 = -S / B2;
                p3 = 2.0 * A1 * inv_b;
            }
        }
        // the partials overwrite the horizontal sums, which every thread has
        // finished reading before the barrier above
        if (i < kTS * kTS) {
            part[i] = p1;
            part[kTS * kTS + i] = p2;
            part[2 * kTS * kTS + i] = p3;
        }
    }
    __syncthreads();
    double l1_sum = 0.0, edge_sum = 0.0;
    if (grad != nullptr) {
        const float g_l1 = weights[0], g_ssim = weights[1], g_edge = weights[2];
        // horizontal pass of the partials -> [3][kTS][kTO]
        double* bh = ss;
        for (int i = tid; i < kTS * kTO; i += kLossThreads) {
            const int r = i / kTO, c = i - r * kTO;
            double a0 = 0.0, a1 = 0.0, a2 = 0.0;
#pragma unroll
            for (int k = 0; k < 2 * kR + 1; ++k) {
                const double g = w.g[k];
                const int j = r * kTS + c + k;
                a0 = fma(g, part[j], a0);
                a1 = fma(g, part[kTS * kTS + j], a1);
                a2 = fma(g, part[2 * kTS * kTS + j], a2);
            }
            bh[i] = a0;
            bh[kTS * kTO + i] = a1;
            bh[2 * kTS * kTO + i] = a2;
        }
        __syncthreads();
        for (int i = tid; i < kTO * kTO; i += kLossThreads) {
            const int r = i / kTO, c = i - r * kTO;
            const int gy = Y0 + r, gx = X0 + c;
            if (gy >= H || gx >= W) continue;
            double q1 = 0.0, q2 = 0.0, q3 = 0.0;
#pragma unroll
            for (int k = 0; k < 2 * kR + 1; ++k) {
                const double g = w.g[k];
                const int j = (r + k) * kTO + c;
                q1 = fma(g, bh[j], q1);
                q2 = fma(g, bh[kTS * kTO + j], q2);
                q3 = fma(g, bh[2 * kTS * kTO + j], q3);
            }
            const int li = (r + 2 * kR) * kTI + c + 2 * kR;
            const float xv = sx[li], tv = st[li];
            const int64_t gi = img + (int64_t)gy * W + gx;
            const float dssim = (float)((q1 + 2.0 * (double)xv * q2 + (double)tv * q3) * inv_m);
            float gv = g_ssim * dssim + g_l1 * (float)inv_m * sgnf(xv - tv);
            const float d1 = fabsf(xv - tv);
            l1_sum += d1;
            if (mask != nullptr) {
                const float mv = mask[gi], tev = te[gi];
                edge_sum += mv * fabsf(xv - tev);
                gv += g_edge * (float)inv_m * mv * sgnf(xv - tev);
            }
            grad[gi] = gv;
        }
    } else {
        for (int i = tid; i < kTO * kTO; i += kLossThreads) {
            const int r = i / kTO, c = i - r * kTO;
            const int gy = Y0 + r, gx = X0 + c;
            if (gy >= H || gx >= W) continue;
            const int li = (r + 2 * kR) * kTI + c + 2 * kR;
            const float xv = sx[li], tv = st[li];
            l1_sum += fabsf(xv - tv);
            if (mask != nullptr) {
                const int64_t gi = img + (int64_t)gy * W + gx;
                edge_sum += mask[gi] * fabsf(xv - te[gi]);
            }
        }
    }
    block_add3(l1_sum, s_sum, edge_sum, sums);
}

// grad = g_ssim dssim + g_l1 d(mean l1)/dx + g_edge d(mean edge)/dx from a
// stored d(mean ssim)/dx map (the same float operations as the fused kernel).
__global__ void loss_combine_kernel(const float* __restrict__ x, const float* __restrict__ t,
                                    const float* __restrict__ te, const float* __restrict__ mask,
                                    const float* __restrict__ dssim,
                                    const float* __restrict__ weights, float inv_m, int64_t n,
                                    float* __restrict__ grad) {
    const float g_l1 = weights[0], g_ssim = weights[1], g_edge = weights[2];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float xv = x[i];
        float gv = g_ssim * dssim[i] + g_l1 * inv_m * sgnf(xv - t[i]);
        if (mask != nullptr) gv += g_edge * inv_m * mask[i] * sgnf(xv - te[i]);
        grad[i] = gv;
    }
}

__global__ void tv_kernel(const float* __restrict__ v, int64_t D0, int64_t D1, int64_t D2,
                          float inv_denom, const float* __restrict__ weight,
                          float* __restrict__ grad, double* __restrict__ sum) {
    const int64_t n = D0 * D1 * D2;
    const float g_scale = grad != nullptr ? weight[0] * inv_denom : 0.f;
    float acc = 0.f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = i % D2, j = (i / D2) % D1, z = i / (D1 * D2);
        const float c = v[i];
        float gsum = 0.f;
        if (z + 1 < D0) {
            const float d = v[i + D1 * D2] - c;
            acc += fabsf(d);
            gsum -= sgnf(d);
        }
        if (z > 0) gsum += sgnf(c - v[i - D1 * D2]);
        if (j + 1 < D1) {
            const float d = v[i + D2] - c;
            acc += fabsf(d);
            gsum -= sgnf(d);
        }
        if (j > 0) gsum += sgnf(c - v[i - D2]);
        if (k + 1 < D2) {
            const float d = v[i + 1] - c;
            acc += fabsf(d);
            gsum -= sgnf(d);
        }
        if (k > 0) gsum += sgnf(c - v[i - 1]);
        if (grad != nullptr) grad[i] = g_scale * gsum;
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) atomicAdd(sum, (double)acc);
}

}  // namespace

}  // namespace r2s

using namespace r2s;

extern "C" int r2s_projection_loss_f32(const float* renders, const float* targets,
                                       const float* edge_targets, const float* edge_mask,
                                       int64_t C, int64_t H, int64_t W, int window_size,
                                       const float* window_1d, const float* weights, float* grad,
                                       double* sums, r2s_stream_t stream) {
    R2S_REQUIRE(C >= 0 && H >= 0 && W >= 0, "projection_loss: negative size");
    R2S_REQUIRE(window_size == 2 * kR + 1,
                "projection_loss: only the 11-pixel SSIM window of the reference configs is "
                "built");
    R2S_REQUIRE(H < 65536 * kTO && W < 65536 * kTO && C <= 65535, "projection_loss: too large");
    R2S_REQUIRE(sums != nullptr, "projection_loss: null sums");
    R2S_REQUIRE(edge_mask == nullptr || edge_targets != nullptr,
                "projection_loss: edge mask without edge targets");
    R2S_REQUIRE(grad == nullptr || weights != nullptr, "projection_loss: gradient without weights");
    if (C * H * W == 0) return R2S_OK;
    R2S_REQUIRE(renders && targets, "projection_loss: null image");
    // 1-D weights of the reference window (metric.py:14-18): exp(-(x - 5)^2 / 4.5),
    // normalized, float32.  SSIM on smooth images depends on the window's sum
    // to ~1e-7, so a caller that has the reference's own float32 weights
    // passes them (host array of 11 floats); otherwise they are normalized here.
    Window11 w;
    if (window_1d != nullptr) {
        for (int k = 0; k < 2 * kR + 1; ++k) w.g[k] = (double)window_1d[k];
    } else {
        double e[2 * kR + 1], tot = 0.0;
        for (int k = 0; k < 2 * kR + 1; ++k) {
            e[k] = std::exp(-double((k - kR) * (k - kR)) / (2.0 * 1.5 * 1.5));
            tot += e[k];
        }
        for (int k = 0; k < 2 * kR + 1; ++k) w.g[k] = (double)(float)(e[k] / tot);
    }
    if (int rc = set_dynamic_smem(proj_loss_kernel, kLossSmem, "projection_loss")) return rc;
    const dim3 grid((unsigned)((W + kTO - 1) / kTO), (unsigned)((H + kTO - 1) / kTO), (unsigned)C);
    proj_loss_kernel<<<grid, kLossThreads, kLossSmem, stream>>>(
        renders, targets, edge_targets, edge_mask, (int)H, (int)W, w, 0.01 * 0.01, 0.03 * 0.03,
        weights, 1.0 / double(C * H * W), grad, sums);
    return check_launch("projection_loss");
}

extern "C" int r2s_tv_loss_f32(const float* volume, int64_t D0, int64_t D1, int64_t D2,
                               const float* weight, float* grad, double* sum,
                               r2s_stream_t stream) {
    R2S_REQUIRE(D0 >= 0 && D1 >= 0 && D2 >= 0, "tv_loss: negative size");
    R2S_REQUIRE(sum != nullptr, "tv_loss: null sum");
    R2S_REQUIRE(grad == nullptr || weight != nullptr, "tv_loss: gradient without weight");
    const int64_t n = D0 * D1 * D2;
    if (n == 0) return R2S_OK;
    R2S_REQUIRE(volume != nullptr, "tv_loss: null volume");
    const int64_t denom = (D0 - 1) * D1 * D2 + D0 * (D1 - 1) * D2 + D0 * D1 * (D2 - 1);
    const double inv = 1.0 / (double)(denom > 1 ? denom : 1);
    const int64_t blocks = std::min<int64_t>((n + kThreads - 1) / kThreads, 148 * 32);
    tv_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(volume, D0, D1, D2, (float)inv, weight,
                                                         grad, sum);
    return check_launch("tv_loss");
}

extern "C" int r2s_projection_loss_combine_f32(const float* renders, const float* targets,
                                               const float* edge_targets, const float* edge_mask,
                                               const float* dssim, int64_t n, const float* weights,
                                               float* grad, r2s_stream_t stream) {
    R2S_REQUIRE(n >= 0, "projection_loss_combine: negative size");
    if (n == 0) return R2S_OK;
    R2S_REQUIRE(renders && targets && dssim && weights && grad,
                "projection_loss_combine: null pointer");
    R2S_REQUIRE(edge_mask == nullptr || edge_targets != nullptr,
                "projection_loss_combine: edge mask without edge targets");
    const int64_t blocks = std::min<int64_t>((n + kThreads - 1) / kThreads, 148 * 32);
    loss_combine_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(
        renders, targets, edge_targets, edge_mask, dssim, weights, (float)(1.0 / double(n)), n,
        grad);
    return check_launch("projection_loss_combine");
}
