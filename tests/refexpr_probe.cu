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

// 3D: one Gaussian per 16^3 cell of a [16 ncz, 16 ncy, 16 ncx] volume;
// out[c, z, y, x] = alpha of voxel (x, y, z) of Gaussian c's own cell, 0 where
// the expression drops the pair.
__global__ void probe3d_kernel(int variant, const float* means3d, const float* conics,
                               const float* opac, const int* cells, int C, float* out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)C * 4096) return;
    const int c = (int)(i >> 12), v = (int)(i & 4095);
    const int z = v >> 8, y = (v >> 4) & 15, x = v & 15;
    const float d1 = ((float)(cells[3 * c] + x) + 0.5f) - means3d[3 * c];
    const float d2 = ((float)(cells[3 * c + 1] + y) + 0.5f) - means3d[3 * c + 1];
    const float d3 = ((float)(cells[3 * c + 2] + z) + 0.5f) - means3d[3 * c + 2];
    out[i] = r2s::ref_alpha3d(variant, conics + 6 * c, opac[c], d1, d2, d3);
}

extern "C" __attribute__((visibility("default"))) int probe_alpha3d(int variant, const float* means3d,
                             const float* conics, const float* opac, const int* cells, int C,
                             float* out, void* stream) {
    const long long n = (long long)C * 4096;
    probe3d_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        variant, means3d, conics, opac, cells, C, out);
    return (int)cudaGetLastError();
}
