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
