// Test probe: evaluates the restated cut-off expressions of
// bt-3dgs_b200/csrc/r2s_refexpr.cuh over whole images, one Gaussian per
// image, for tests/test_gpu_refexpr.py (compiled there with the library's
// nvcc flags).  out[c, i, j] = alpha of pixel (i, j) of image c, 0 where the
// expression drops the pair.
#include <cuda_runtime.h>

#include "../bt-3dgs_b200/csrc/r2s_refexpr.cuh"

__global__ void probe_kernel(int variant, const float* means2d, const float* conics,
                             const float* wmu, int C, int W, int H, float* out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)C * W * H) return;
    const int c = (int)(i / ((long long)W * H));
    const int p = (int)(i - (long long)c * W * H);
    const int y = p / W, x = p - y * W;
    const float dx = ((float)x + 0.5f) - means2d[2 * c];
    const float dy = ((float)y + 0.5f) - means2d[2 * c + 1];
    out[i] = r2s::ref_alpha2d(variant, conics[3 * c], conics[3 * c + 1], conics[3 * c + 2],
                              wmu[c], dx, dy);
}

extern "C" __attribute__((visibility("default"))) int probe_alpha2d(int variant, const float* means2d, const float* conics,
                             const float* wmu, int C, int W, int H, float* out, void* stream) {
    const long long n = (long long)C * W * H;
    probe_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        variant, means2d, conics, wmu, C, W, H, out);
    return (int)cudaGetLastError();
}
