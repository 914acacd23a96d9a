// Pipe-throughput calibration kernels (measurement support, not on the path).
//
// The rasterizer and voxelizer kernels of this library are bound by the SM's
// FP32 (FMA) pipe and its MUFU ex2 unit, not by HBM or the tensor cores.  To
// report their roofline fractions against what this GPU delivers at the
// clock it runs at, the benchmark times these two kernels with CUDA events
// beside the hot path:
//   * r2s_calib_ffma_f32: every thread runs kChains independent FFMA chains
//     (x = x * a + b) for `iters` steps: 2 FLOP per FFMA;
//   * r2s_calib_ex2_f32:  every thread runs kChains independent ex2.approx
//     chains (x = 2^(x * m), one FMUL feeding each ex2 so that the values stay
//     in range; the FMUL rides on the FMA pipe, which has 8x the MUFU rate).
// Enough chains per thread and enough resident warps hide the pipes'
// latencies, so the rate is the issue/pipe peak.  The results are written to
// `out` (one float per thread) so the compiler cannot drop the chains.
#include "r2s_common.cuh"

namespace r2s {
namespace {

constexpr int kCalibThreads = 256;
constexpr int kChains = 8;

__global__ void __launch_bounds__(kCalibThreads)
calib_ffma_kernel(float* __restrict__ out, int64_t iters, float a, float b) {
    float x[kChains];
#pragma unroll
    for (int k = 0; k < kChains; ++k) x[k] = (float)(threadIdx.x + k) * 1e-3f;
    for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
        for (int k = 0; k < kChains; ++k) x[k] = fmaf(x[k], a, b);
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kChains; ++k) s += x[k];
    out[(int64_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(kCalibThreads)
calib_ex2_kernel(float* __restrict__ out, int64_t iters, float m) {
    float x[kChains];
#pragma unroll
    for (int k = 0; k < kChains; ++k) x[k] = -(float)(threadIdx.x + k) * 1e-3f;
    for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
        for (int k = 0; k < kChains; ++k) x[k] = ex2_approx(x[k] * m);
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kChains; ++k) s += x[k];
    out[(int64_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

int calib_args(const float* out, int64_t iters, int blocks) {
    R2S_REQUIRE(out != nullptr, "calibration: out is null");
    R2S_REQUIRE(iters > 0 && blocks > 0, "calibration: iters and blocks must be positive");
    return R2S_OK;
}

}  // namespace
}  // namespace r2s

extern "C" int r2s_calib_ffma_f32(float* out, int64_t iters, int blocks, r2s_stream_t stream) {
    if (int rc = r2s::calib_args(out, iters, blocks)) return rc;
    r2s::calib_ffma_kernel<<<blocks, r2s::kCalibThreads, 0, (cudaStream_t)stream>>>(
        out, iters, 0.999f, 1e-3f);
    return r2s::check_launch("calib_ffma");
}

extern "C" int r2s_calib_ex2_f32(float* out, int64_t iters, int blocks, r2s_stream_t stream) {
    if (int rc = r2s::calib_args(out, iters, blocks)) return rc;
    r2s::calib_ex2_kernel<<<blocks, r2s::kCalibThreads, 0, (cudaStream_t)stream>>>(
        out, iters, -0.5f);
    return r2s::check_launch("calib_ex2");
}
